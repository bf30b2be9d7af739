"""transformers Qwen3-MoE smoke test with the fused EP blocks (reference: scripts/hf_qwen.py).

Builds a random-init transformers Qwen3MoeForCausalLM (or loads ``--model-path`` when a
local checkpoint exists), swaps every sparse MoE block for ``SepxQwen3MoeBlock`` and runs
greedy ``generate``. Without a tokenizer it prompts with token ids; with one it uses a
neutral prompt. Single GPU.

    python examples/hf_qwen.py [--model-path /path/to/Qwen3-30B-A3B] [--max-new-tokens 32]
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from spec_ep.integrations.hf_qwen import random_hf_model, swap_moe_blocks  # noqa: E402
from spec_ep.parallel.ep import ExpertParallel  # noqa: E402

PROMPT = "Explain expert parallelism in one short paragraph."


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-path", default=None)
    ap.add_argument("--max-new-tokens", type=int, default=32)
    args = ap.parse_args()
    tok = None
    if args.model_path and os.path.isdir(args.model_path):
        from transformers import AutoModelForCausalLM, AutoTokenizer

        model = AutoModelForCausalLM.from_pretrained(args.model_path, dtype=torch.bfloat16).cuda().eval()
        tok = AutoTokenizer.from_pretrained(args.model_path)
    else:
        model = random_hf_model().cuda().eval()
    c = model.config
    ep = ExpertParallel(c.num_experts, c.num_experts_per_tok, c.hidden_size, max_tokens=4096)
    print(f"swapped {swap_moe_blocks(model, ep)} MoE blocks")
    if tok is not None:
        inputs = tok.apply_chat_template([{"role": "user", "content": PROMPT}], add_generation_prompt=True,
                                         return_tensors="pt", return_dict=True).to("cuda")
    else:
        inputs = {"input_ids": torch.randint(0, c.vocab_size, (1, 16), device="cuda")}
    with torch.inference_mode():
        out = model.generate(**inputs, max_new_tokens=args.max_new_tokens, do_sample=False)
    gen = out[0][inputs["input_ids"].shape[-1]:]
    print(tok.decode(gen, skip_special_tokens=True) if tok is not None else gen.tolist())
    ep.check()
    ep.close()


if __name__ == "__main__":
    main()
