"""The allocation-free permutation entry point, called through its exported C symbol.

Some callers cannot allocate GPU memory when they call us (allocator callbacks,
runtimes that fix their device-memory budget up front, C/FFI hosts without the PyTorch
allocator). ``sepx_moe_permute_noalloc`` serves them: it keeps its temporaries in a
static device array of the library. This test calls it through ctypes and checks that
two calls in a row give exactly the layout the allocating expert-parallel dispatch
(``ExpertParallel.dispatch_fwd`` at world size 1) produces. The file is named so that
pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry():
    import spec_ep._C as ext  # loads the library (and its torch dependencies) first

    lib = ctypes.CDLL(ext.__file__)
    f = lib.sepx_moe_permute_noalloc
    f.restype = ctypes.c_int
    P, I = ctypes.c_void_p, ctypes.c_int
    f.argtypes = [P, P, P, I, I, I, I, P, I, P, P, P, P, P, P]
    return f


def _routing(T, E, k, H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    logits = torch.randn(T, E, device="cuda", generator=g)
    logits[:, : E // 4] += 1.5  # skewed: a quarter of the experts are hot
    w, e = torch.softmax(logits, -1).topk(k, -1)
    return x, e.int().contiguous(), (w / w.sum(-1, keepdim=True)).contiguous()


@pytest.mark.parametrize("T,E,k,H", [(2048, 64, 8, 512), (8192, 256, 8, 256)])
def test_noalloc_permute_matches_allocating_dispatch_twice(T, E, k, H):
    """Two calls in a row, at a mid size and at the scratch array's limits (T = 8192,
    E = 256), give the allocating dispatch's layout."""
    from spec_ep.parallel.ep import ExpertParallel

    f = _entry()
    ep = ExpertParallel(E, k, H, max_tokens=T)
    R = ep.cap_rows
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((0, 1)):
        x, te, tw = _routing(T, E, k, H, seed)
        st = ep.dispatch_fwd(x, te, tw)
        xp = torch.empty(R, H, device="cuda", dtype=torch.bfloat16)
        go = torch.empty(E + 1, device="cuda", dtype=torch.int32)
        rw = torch.empty(R, device="cuda", dtype=torch.float32)
        rs = torch.empty(R, device="cuda", dtype=torch.int32)
        inv = torch.empty(T, k, device="cuda", dtype=torch.int32)
        status = torch.full((1,), -1, device="cuda", dtype=torch.int32)
        rc = f(x.data_ptr(), te.data_ptr(), tw.data_ptr(), T, k, H, E, xp.data_ptr(), R, go.data_ptr(),
               rw.data_ptr(), rs.data_ptr(), inv.data_ptr(), status.data_ptr(), stream)
        assert rc == 0, f"call {call}: return code {rc}"
        torch.cuda.synchronize()
        ep.check()
        assert status.item() == 0
        assert torch.equal(go, st.group_off)
        n = int(go[-1])
        assert n >= T * k
        # pure data movement: the two paths must agree exactly
        assert torch.equal(xp[:n], st.xp[:n])
        assert torch.equal(rw[:n], st.row_w[:n])
        assert torch.equal(rs[:n], st.row_src[:n])
        assert torch.equal(inv, st.inv_rows[0])
    ep.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    f = _entry()
    stream = torch.cuda.current_stream().cuda_stream
    dummy = torch.empty(16, device="cuda")
    p = dummy.data_ptr()
    assert f(p, p, p, 8193, 8, 512, 64, p, 10**7, p, p, p, p, p, stream) == 1
    assert f(p, p, p, 1024, 9, 512, 64, p, 10**7, p, p, p, p, p, stream) == 2
    assert f(p, p, p, 1024, 8, 512, 257, p, 10**7, p, p, p, p, p, stream) == 3
    assert f(p, p, p, 1024, 8, 500, 64, p, 10**7, p, p, p, p, p, stream) == 4
    assert f(p, p, p, 1024, 8, 512, 64, p, 1024, p, p, p, p, p, stream) == 5
    # rows move as 16-byte vectors: a misaligned x or xp is refused before any launch
    assert f(p + 2, p, p, 1024, 8, 512, 64, p, 10**7, p, p, p, p, p, stream) == 8
    assert f(p, p, p, 1024, 8, 512, 64, p + 8, 10**7, p, p, p, p, p, stream) == 8


def test_noalloc_out_of_range_and_masked_expert_ids():
    """An id >= E is reported (status 5) and dropped; an id of -1 is dropped silently;
    every other choice is placed exactly as in a call without the bad entries."""
    f = _entry()
    T, E, k, H = 256, 16, 4, 64
    x, te, tw = _routing(T, E, k, H, seed=3)
    bad = te.clone()
    bad[5, 1] = E + 3   # out of range: reported
    bad[9, 2] = -1      # masked: silent
    R = T * k + 64 * E
    stream = torch.cuda.current_stream().cuda_stream

    def run(ids):
        xp = torch.empty(R, H, device="cuda", dtype=torch.bfloat16)
        go = torch.empty(E + 1, device="cuda", dtype=torch.int32)
        rw = torch.empty(R, device="cuda", dtype=torch.float32)
        rs = torch.empty(R, device="cuda", dtype=torch.int32)
        inv = torch.empty(T, k, device="cuda", dtype=torch.int32)
        status = torch.full((1,), -1, device="cuda", dtype=torch.int32)
        rc = f(x.data_ptr(), ids.data_ptr(), tw.data_ptr(), T, k, H, E, xp.data_ptr(), R, go.data_ptr(),
               rw.data_ptr(), rs.data_ptr(), inv.data_ptr(), status.data_ptr(), stream)
        assert rc == 0
        torch.cuda.synchronize()
        return int(status.item()), inv, go, rs, xp

    st_bad, inv_bad, go_bad, rs_bad, xp_bad = run(bad)
    assert st_bad == 5
    assert int(inv_bad[5, 1]) == -1 and int(inv_bad[9, 2]) == -1
    masked = bad.clone()
    masked[5, 1] = -1  # the same routing with the bad entry masked instead
    st_m, inv_m, go_m, rs_m, xp_m = run(masked)
    assert st_m == 0
    assert torch.equal(inv_bad, inv_m) and torch.equal(go_bad, go_m)
    n = int(go_m[-1])
    cnt = bad[(bad >= 0) & (bad < E)].long().bincount(minlength=E)
    assert n == int(((cnt + 63) // 64 * 64).sum())
    assert torch.equal(rs_bad[:n], rs_m[:n]) and torch.equal(xp_bad[:n], xp_m[:n])
