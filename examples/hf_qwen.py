"""transformers Qwen3-MoE smoke test with the fused EP blocks (reference: scripts/hf_qwen.py).

Builds a transformers Qwen3MoeForCausalLM, swaps every sparse MoE block for
``SepxQwen3MoeBlock`` and runs greedy ``generate``. As in the reference, the model is
random-init from the checkpoint's config unless ``--load-weights`` is given; without a
local ``--model-path`` it is a small random Qwen3-MoE. Without a tokenizer it prompts
with token ids; with one it uses a neutral prompt. Single GPU.

    python examples/hf_qwen.py [--model-path /path/to/Qwen3-30B-A3B [--load-weights]] [--max-new-tokens 32]
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from spec_ep.integrations.hf_qwen import random_hf_model, swap_moe_blocks  # noqa: E402
from spec_ep.parallel.ep import ExpertParallel  # noqa: E402

PROMPT = "Explain expert parallelism in one short paragraph."


def build_model(model_path=None, load_weights=False):
    """(model, tokenizer or None) on the host: the checkpoint's weights with
    ``load_weights``, else its config with random weights (the reference's default,
    scripts/hf_qwen.py:26-42); a small random Qwen3-MoE without a local path."""
    if not (model_path and os.path.isdir(model_path)):
        if load_weights:
            raise SystemExit("--load-weights needs --model-path with a local checkpoint")
        return random_hf_model(), None
    from transformers import AutoConfig, AutoModelForCausalLM, AutoTokenizer

    if load_weights:
        model = AutoModelForCausalLM.from_pretrained(model_path, dtype=torch.bfloat16)
    else:
        model = AutoModelForCausalLM.from_config(AutoConfig.from_pretrained(model_path), dtype=torch.bfloat16)
    # only a checkpoint that ships tokenizer files has a tokenizer (transformers would
    # otherwise build an empty one from the model type)
    files = ("tokenizer.json", "tokenizer_config.json", "vocab.json", "tokenizer.model")
    has_tok = any(os.path.exists(os.path.join(model_path, f)) for f in files)
    tok = AutoTokenizer.from_pretrained(model_path) if has_tok else None
    return model, tok


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-path", default=None)
    ap.add_argument("--load-weights", action="store_true",
                    help="load the checkpoint's weights (default: its config with random weights)")
    ap.add_argument("--max-new-tokens", type=int, default=32)
    args = ap.parse_args()
    model, tok = build_model(args.model_path, args.load_weights)
    model = model.cuda().eval()
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
