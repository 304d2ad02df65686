"""gr_bd_attention_noalloc: the attention entry point for callers that cannot allocate device memory (a host whose
allocator owns the device-memory budget, or code running under stream capture).  It must give the same output as
gr_bd_attention with a caller-provided workspace, also on back-to-back calls that reuse the library's fixed scratch
array, and it must refuse work that does not fit that array.

This file is collected last on purpose: it runs after every other test and also passes alone in a fresh process."""
import math

import pytest
import torch

from gravityocr_b200 import _lib as L

pytestmark = pytest.mark.gpu
DEV = "cuda"
NQ, NKV, D, PS = 16, 8, 128, 16


def _case(seed, bs, K, draft, max_prefix):
    g = torch.Generator().manual_seed(seed)
    S = torch.randint(200, max_prefix, (bs,), generator=g)
    base_add = 0 if draft else 1
    need = [(int(s) + base_add + K + PS - 1) // PS for s in S]
    P = max(need)
    n_pages = sum(need) + 4
    perm = torch.randperm(n_pages, generator=g).to(torch.int32)
    pt = torch.zeros((bs, P), dtype=torch.int32)
    o = 0
    for b in range(bs):
        pt[b, : need[b]] = perm[o: o + need[b]]
        o += need[b]
    kc = torch.randn((n_pages, NKV, PS, D), generator=g).to(DEV, torch.bfloat16)
    vc = torch.randn((n_pages, NKV, PS, D), generator=g).to(DEV, torch.bfloat16)
    q = torch.randn((bs * K, NQ, D), generator=g).to(DEV, torch.bfloat16)
    return q, kc, vc, pt.to(DEV), S.to(DEV), base_add


def _with_workspace(q, kc, vc, pt, seq, bs, K, draft, base_add, chunk, splits):
    ws = torch.zeros((L.attention_workspace_bytes(bs, K, NQ, NKV, splits),), dtype=torch.uint8, device=DEV)
    out = torch.zeros((bs * K, NQ, D), dtype=torch.bfloat16, device=DEV)
    L.bd_attention(q, kc, vc, pt, seq, bs, K, draft, base_add, NQ, NKV, PS, chunk, splits, out, ws)
    return out


def _compare(seed, bs, K, draft, chunk, max_prefix, want_global):
    q, kc, vc, pt, seq, base_add = _case(seed, bs, K, draft, max_prefix)
    splits = int(math.ceil((int(seq.max()) + base_add + K) / chunk))
    assert splits > 1
    # more CTAs than SMs: the splits merge through the scratch (partials and tickets); at most one CTA per SM, they
    # merge inside a thread-block cluster and the scratch is not touched
    assert (bs * NKV * splits > L.num_sms()) == want_global
    assert L.attention_workspace_bytes(bs, K, NQ, NKV, splits) <= L.NOALLOC_SCRATCH_BYTES
    ref = _with_workspace(q, kc, vc, pt, seq, bs, K, draft, base_add, chunk, splits)
    out = torch.full_like(ref, float("nan"))
    st = torch.zeros((1,), dtype=torch.int32, device=DEV)
    L.bd_attention_noalloc(q, kc, vc, pt, seq, bs, K, draft, base_add, NQ, NKV, PS, chunk, splits, out, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    # same kernel, same split points, same merge order: identical (the attention tests' tolerance would be rtol 2e-2)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("tc_mode", [1, 0])
def test_noalloc_attention_matches_workspace_version_twice_in_a_row(tc_mode):
    """Two calls of different shapes back to back whose splits merge through the fixed array: the second call finds
    the first call's partials and tickets there.  Mode 1 runs the tcgen05 kernel on these grids, mode 0 the mma.sync
    kernel; both merge through global scratch."""
    L.set_attention_tc(tc_mode)
    try:
        _compare(5, 5, 17, True, 256, 1700, want_global=True)     # 5 x 8 x 6 = 240 CTAs, 5.8 MiB of scratch
        _compare(6, 4, 33, False, 192, 1100, want_global=True)    # 4 x 8 x 6 = 192 CTAs, 7.7 MiB
        _compare(7, 5, 17, False, 192, 1450, want_global=True)    # 240 CTAs, 5.8 MiB
    finally:
        L.set_attention_tc(1)


def test_noalloc_attention_small_grids():
    # grids of at most one CTA per SM merge inside a cluster; the call must still match
    for seed, bs, K, draft, chunk in [(5, 3, 17, True, 256), (6, 2, 33, False, 256)]:
        _compare(seed, bs, K, draft, chunk, 1500, want_global=False)


def test_noalloc_attention_refuses_work_beyond_its_array():
    bs, K, chunk = 64, 17, 64
    splits = 64   # 64 requests x 8 heads x 64 splits of partials is far more than 8 MiB
    assert L.attention_workspace_bytes(bs, K, NQ, NKV, splits) > L.NOALLOC_SCRATCH_BYTES
    q = torch.zeros((bs * K, NQ, D), dtype=torch.bfloat16, device=DEV)
    kc = torch.zeros((4, NKV, PS, D), dtype=torch.bfloat16, device=DEV)
    pt = torch.zeros((bs, 4), dtype=torch.int32, device=DEV)
    seq = torch.zeros((bs,), dtype=torch.int64, device=DEV)
    out = torch.zeros_like(q)
    with pytest.raises(RuntimeError, match="8 MiB"):
        L.bd_attention_noalloc(q, kc, kc, pt, seq, bs, K, True, 0, NQ, NKV, PS, chunk, splits, out)
