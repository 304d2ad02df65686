"""Kernel-level parity on a B200: every CUDA kernel through the C ABI against a plain fp32 PyTorch reference of the
same op (floating point, tolerance stated per test) or the CPU oracle (integer work, bit-exact)."""
import json
import math
import os

import numpy as np
import pytest
import torch

from gravityocr_b200 import _lib as L
from gravityocr_b200.config import ModelConfig
from gravityocr_b200.engine import rope_inv_freq

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ws(n_out, k_in, m, splits=0):
    # room for whichever epilogue mode the call plans (the split count depends on it)
    modes = (L.EPI_STORE_F32, L.EPI_STORE_BF16, L.EPI_SWIGLU, L.EPI_QKV_ROPE, L.EPI_ARGMAX, L.EPI_PARTIAL_F32)
    sps = [splits] if splits else [L.linear_default_splits(n_out, k_in, m, md) for md in modes]
    return torch.zeros((max(L.linear_workspace_bytes(n_out, m, sp) for sp in sps),), dtype=torch.uint8, device=DEV)


def _rand(shape, g, scale=1.0, dtype=torch.bfloat16):
    return (torch.randn(shape, generator=g) * scale).to(DEV, dtype)


# large m: several token tiles per weight tile (cost-model tiling); odd m: a ragged last token tile, whose units run
# after the full tiles' at a narrower MMA N (1088 rows -> 4 x 256 + 64; 513 -> 2 x 256 + 1; 272 -> 224 + 48)
SHAPES = [(1536, 2048, 17), (4096, 1536, 17), (9216, 1536, 34), (1536, 4608, 17), (1536, 1536, 5),
          (4096, 1536, 1088), (1536, 2048, 300), (1536, 4608, 2176), (256, 128, 1), (1536, 4608, 64),
          (4096, 1536, 129), (9216, 1536, 513), (1152, 1536, 300), (9216, 1536, 1088), (4096, 1536, 272),
          (1536, 4608, 272)]


@pytest.mark.parametrize("n_out,k_in,m", SHAPES)
def test_linear_store_f32(n_out, k_in, m):
    g = torch.Generator().manual_seed(n_out * 7 + k_in * 3 + m)
    w = _rand((n_out, k_in), g, 0.02)
    x = _rand((m, k_in), g)
    out = torch.full((m, n_out), float("nan"), device=DEV)
    e = L.Epilogue()
    e.mode, e.out, e.ld_out = L.EPI_STORE_F32, out.data_ptr(), n_out
    st = torch.zeros((1,), dtype=torch.int32, device=DEV)
    L.linear(w, x, m, e, _ws(n_out, k_in, m), status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ref = x.float() @ w.float().T
    # fp32 accumulation of bf16 products in another order: |err| ~ 1e-6 * |sum of |terms||
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=2e-4 * math.sqrt(k_in))


@pytest.mark.parametrize("n_out,k_in,m,ld_extra", [(1536, 2048, 17, 0), (4096, 1536, 300, 8), (1536, 1536, 1088, 0)])
def test_linear_store_bf16(n_out, k_in, m, ld_extra):
    """bf16 store epilogue (16-byte vector stores through shared memory), also into a wider row (ld_out > n_out)."""
    g = torch.Generator().manual_seed(n_out + m)
    w = _rand((n_out, k_in), g, 0.02)
    x = _rand((m, k_in), g)
    ld = n_out + ld_extra
    out = torch.full((m, ld), float("nan"), dtype=torch.bfloat16, device=DEV)
    e = L.Epilogue()
    e.mode, e.out, e.ld_out = L.EPI_STORE_BF16, out.data_ptr(), ld
    L.linear(w, x, m, e, _ws(n_out, k_in, m))
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T
    torch.testing.assert_close(out[:, :n_out].float(), ref, rtol=1e-2, atol=1e-2)
    if ld_extra:
        assert torch.isnan(out[:, n_out:].float()).all()  # nothing written past the tile


@pytest.mark.parametrize("splits", [1, 2, 4, 8])
def test_linear_splits_agree(splits):
    n_out, k_in, m = 1536, 2048, 17
    g = torch.Generator().manual_seed(5)
    w, x = _rand((n_out, k_in), g, 0.02), _rand((m, k_in), g)
    out = torch.zeros((m, n_out), device=DEV)
    e = L.Epilogue()
    e.mode, e.out, e.ld_out = L.EPI_STORE_F32, out.data_ptr(), n_out
    ws = torch.zeros((L.linear_workspace_bytes(n_out, m, splits),), dtype=torch.uint8, device=DEV)
    for _ in range(2):  # the second call reuses re-armed tickets
        out.zero_()
        L.linear(w, x, m, e, ws, splits=splits)
    torch.cuda.synchronize()
    torch.testing.assert_close(out, x.float() @ w.float().T, rtol=1e-3, atol=1e-2)
    assert int(ws[:256].view(torch.int32).abs().sum().item()) == 0


@pytest.mark.parametrize("m", [17, 136, 1088])
def test_linear_swiglu(m):
    I, H = 4608, 1536
    g = torch.Generator().manual_seed(m)
    w = _rand((2 * I, H), g, 0.02)
    x = _rand((m, H), g)
    wp = torch.empty_like(w)
    L.pack_gate_up(w, wp, I)
    act = torch.zeros((m, I), dtype=torch.bfloat16, device=DEV)
    e = L.Epilogue()
    e.mode, e.out, e.ld_out = L.EPI_SWIGLU, act.data_ptr(), I
    L.linear(wp, x, m, e, _ws(2 * I, H, m))
    torch.cuda.synchronize()
    gu = x.float() @ w.float().T
    ref = gu[:, I:] * torch.nn.functional.silu(gu[:, :I])
    torch.testing.assert_close(act.float(), ref, rtol=2e-2, atol=2e-3)


def _rope_ref(x, pos, inv_freq, rd):
    # the angle is the fp32 product pos * inv_freq (as the reference computes it); cos / sin in x's precision
    f = (pos.float()[:, None] * inv_freq.float()[None, :]).to(x.dtype)
    c, s = f.cos()[:, None, :], f.sin()[:, None, :]
    out = x.clone()
    x0, x1 = x[..., 0:rd:2], x[..., 1:rd:2]
    out[..., 0:rd:2] = x0 * c - x1 * s
    out[..., 1:rd:2] = x1 * c + x0 * s
    return out


@pytest.mark.parametrize("m,max_pos", [(17, 8000), (170, 8000), (1088, 8000), (1088, 65536)])
def test_linear_qkv_rope_kvwrite(m, max_pos):
    """Q/K/V projection with the RoPE epilogue (cos / sin computed in registers) and the paged K/V write."""
    cfg = ModelConfig()
    g = torch.Generator().manual_seed(11 + m)
    H, nq, nkv, D = cfg.hidden, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    w = _rand((cfg.qkv_dim, H), g, 0.02)
    x = _rand((m, H), g)
    n_pages, ps = m // 16 + 64, 16
    pos = torch.randint(0, max_pos, (m,), generator=g, dtype=torch.int32)
    perm = torch.randperm(n_pages * ps, generator=g)[:m]
    slots = perm.to(torch.int64)
    kc = torch.zeros((n_pages, nkv, ps, D), dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.zeros((m, nq * D), dtype=torch.bfloat16, device=DEV)
    inv = rope_inv_freq(cfg).to(DEV)
    pos_d, slots_d = pos.to(DEV), slots.to(DEV)
    e = L.Epilogue()
    e.mode = L.EPI_QKV_ROPE
    e.q_out, e.k_cache, e.v_cache = q.data_ptr(), kc.data_ptr(), vc.data_ptr()
    e.row_pos, e.row_slot, e.inv_freq = pos_d.data_ptr(), slots_d.data_ptr(), inv.data_ptr()
    e.rotary_dim, e.n_q_heads, e.n_kv_heads, e.page_size = cfg.rotary_dim, nq, nkv, ps
    L.linear(w, x, m, e, _ws(cfg.qkv_dim, H, m))
    torch.cuda.synchronize()
    y = x.float() @ w.float().T
    qr = _rope_ref(y[:, : nq * D].view(m, nq, D), pos_d, inv, cfg.rotary_dim)
    kr = _rope_ref(y[:, nq * D: (nq + nkv) * D].view(m, nkv, D), pos_d, inv, cfg.rotary_dim)
    vr = y[:, (nq + nkv) * D:].view(m, nkv, D)
    torch.testing.assert_close(q.float().view(m, nq, D), qr, rtol=2e-2, atol=2e-2)
    kg = kc.view(n_pages * 0 + n_pages, nkv, ps, D).permute(0, 2, 1, 3).reshape(n_pages * ps, nkv, D)[slots_d]
    vg = vc.permute(0, 2, 1, 3).reshape(n_pages * ps, nkv, D)[slots_d]
    torch.testing.assert_close(kg.float(), kr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(vg.float(), vr, rtol=2e-2, atol=2e-2)
    # The rotation itself to one bf16 ulp: the fp64 rotation of the kernel's own unrotated values (v heads carry the
    # same GEMM; here the q projection is recomputed in fp64 from the bf16 inputs) rounds to within 1 ulp of q.
    y64 = x.double() @ w.double().T
    q64 = _rope_ref(y64[:, : nq * D].view(m, nq, D), pos_d, inv, cfg.rotary_dim)
    ulp = torch.finfo(torch.bfloat16).eps * q64.abs().clamp_min(1e-3)
    assert ((q.double().view(m, nq, D) - q64).abs() <= 1.01 * ulp + 1e-4).all()


@pytest.mark.parametrize("m", [17, 34, 300, 1088])
def test_linear_argmax(m):
    V, H = 59392, 1536
    g = torch.Generator().manual_seed(23 + m)
    w = _rand((V, H), g, 0.02)
    x = _rand((m, H), g)
    idx = torch.full((m,), -1, dtype=torch.int32, device=DEV)
    top = torch.zeros((m,), device=DEV)
    gap = torch.zeros((m,), device=DEV)
    e = L.Epilogue()
    e.mode, e.out_idx, e.out_top1, e.out_gap = L.EPI_ARGMAX, idx.data_ptr(), top.data_ptr(), gap.data_ptr()
    ws = _ws(V, H, m)
    for _ in range(2):
        L.linear(w, x, m, e, ws)
    torch.cuda.synchronize()
    lg = x.float() @ w.float().T
    t2 = torch.topk(lg, 2, dim=-1)
    ref_idx, ref_gap = t2.indices[:, 0], t2.values[:, 0] - t2.values[:, 1]
    sure = ref_gap > 1e-3
    assert torch.equal(idx.long()[sure], ref_idx[sure])
    torch.testing.assert_close(top, t2.values[:, 0], rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(gap, ref_gap, rtol=1e-2, atol=2e-3)


# ---------------------------------------------------------------------- attention
def _attn_ref(q, kc, vc, pt, seq_lens, K, draft, base_add, nq, nkv):
    """fp32 reference: q [bs*K, nq, D], caches [pages, nkv, 16, D], page table [bs, P]."""
    bs = pt.shape[0]
    D = q.shape[-1]
    out = torch.zeros((bs * K, nq, D), device=q.device)
    G = nq // nkv
    for b in range(bs):
        base = int(seq_lens[b]) + base_add
        Lmax = base + K
        npg = (Lmax + 15) // 16
        pages = pt[b, :npg].long()
        kk = kc[pages].permute(0, 2, 1, 3).reshape(npg * 16, nkv, D)[:Lmax].float()
        vv = vc[pages].permute(0, 2, 1, 3).reshape(npg * 16, nkv, D)[:Lmax].float()
        qb = q[b * K: (b + 1) * K].float()                               # [K, nq, D]
        j = torch.arange(K, device=q.device)
        lim = torch.where(j == 0, base + 1, base + K) if draft else base + j + 1
        mask = torch.arange(Lmax, device=q.device)[None, :] < lim[:, None]
        kr = kk.repeat_interleave(G, dim=1)
        vr = vv.repeat_interleave(G, dim=1)
        s = torch.einsum("khd,lhd->hkl", qb, kr) / math.sqrt(D)
        s = s.masked_fill(~mask[None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[b * K: (b + 1) * K] = torch.einsum("hkl,lhd->khd", p, vr)
    return out


@pytest.mark.parametrize("bs,K,draft", [(1, 17, True), (1, 17, False), (8, 17, True), (8, 17, False),
                                        (64, 17, True), (64, 17, False), (3, 5, True), (2, 33, False),
                                        (2, 64, False)])
def test_bd_attention(bs, K, draft):
    """Config 1: prefixes uniform in 256..4096 (seed 1), page 16, GQA 16/8, head_dim 128, Q/K/V ~ N(0, 1)."""
    nq, nkv, D, ps = 16, 8, 128, 16
    g = torch.Generator().manual_seed(1)
    S = torch.randint(256, 4097, (bs,), generator=g)
    base_add = 0 if draft else 1
    need = [(int(s) + base_add + K + ps - 1) // ps for s in S]
    P = max(need) + 1
    n_pages = sum(need) + 8
    perm = torch.randperm(n_pages, generator=g)
    pt = torch.zeros((bs, P), dtype=torch.int32)
    o = 0
    for b in range(bs):
        pt[b, : need[b]] = perm[o: o + need[b]].to(torch.int32)
        pt[b, need[b]:] = perm[o]
        o += need[b]
    kc = _rand((n_pages, nkv, ps, D), g)
    vc = _rand((n_pages, nkv, ps, D), g)
    q = _rand((bs * K, nq, D), g)
    pt_d, seq_d = pt.to(DEV), S.to(DEV)
    ref = _attn_ref(q, kc, vc, pt_d, seq_d, K, draft, base_add, nq, nkv)
    Lmax = int(S.max()) + base_add + K
    min_chunk = max(64, -(-(-(-Lmax // 16)) // 64) * 64)   # the merge takes at most 16 splits
    for chunk in sorted({min_chunk, max(min_chunk, 512), 4096}):
        max_splits = int(math.ceil(Lmax / chunk))
        ws = torch.zeros((max(256, L.attention_workspace_bytes(bs, K, nq, nkv, max_splits)),), dtype=torch.uint8,
                         device=DEV)
        out = torch.full((bs * K, nq, D), float("nan"), dtype=torch.bfloat16, device=DEV)
        st = torch.zeros((1,), dtype=torch.int32, device=DEV)
        for _ in range(2):
            L.bd_attention(q, kc, vc, pt_d, seq_d, bs, K, draft, base_add, nq, nkv, ps, chunk, max_splits, out, ws,
                           status=st)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=1.5e-2)
        # a launch order (longest request first) changes scheduling only
        order = torch.argsort(seq_d, descending=True).to(torch.int32)
        out2 = torch.full_like(out, float("nan"))
        L.bd_attention(q, kc, vc, pt_d, seq_d, bs, K, draft, base_add, nq, nkv, ps, chunk, max_splits, out2, ws,
                       status=st, order=order)
        torch.cuda.synchronize()
        assert torch.equal(out2, out)


# ---------------------------------------------------------------------- row-wise kernels
def test_embed_rows_and_residual_norm():
    cfg = ModelConfig()
    g = torch.Generator().manual_seed(3)
    bs, K, H, V = 3, 17, cfg.hidden, cfg.vocab
    E = _rand((V, H), g, 0.02)
    nw = _rand((H,), g, 0.02)
    seeds = torch.randint(0, V, (8,), generator=g).to(DEV)
    rpi = torch.tensor([5, 0, 2], dtype=torch.int64, device=DEV)
    seq = torch.tensor([300, 17, 1000], dtype=torch.int64, device=DEV)
    pt = torch.arange(bs * 80, dtype=torch.int32, device=DEV).view(bs, 80).flip(1).contiguous()
    M = bs * K
    h = torch.zeros((M, H), device=DEV)
    x = torch.zeros((M, H), dtype=torch.bfloat16, device=DEV)
    pos = torch.zeros((M,), dtype=torch.int32, device=DEV)
    slot = torch.zeros((M,), dtype=torch.int64, device=DEV)
    ids = torch.zeros((M,), dtype=torch.int32, device=DEV)
    st = torch.zeros((1,), dtype=torch.int32, device=DEV)
    inv = rope_inv_freq(cfg).to(DEV)
    for mode in (L.ROWS_DRAFT, L.ROWS_VERIFY):
        am = torch.randint(0, V, (M,), generator=g, dtype=torch.int32).to(DEV)
        L.embed_rows(mode, bs, K, seeds=seeds, rpi=rpi, ids32=am, seq_lens=seq, page_table=pt, page_size=16,
                     embed=E, vocab=V, mask_id=cfg.mask_id, norm_w=nw, eps=cfg.rms_eps, h_out=h, x_out=x, row_pos=pos,
                     row_slot=slot, row_ids=ids, status=st)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        j = torch.arange(K, device=DEV).repeat(bs)
        b = torch.arange(bs, device=DEV).repeat_interleave(K)
        if mode == L.ROWS_DRAFT:
            want_ids = torch.where(j == 0, seeds[rpi][b], torch.full_like(j, cfg.mask_id))
            want_pos = seq[b] + j
        else:
            want_ids = am.long()
            want_pos = seq[b] + 1 + j
        assert torch.equal(ids.long(), want_ids)
        assert torch.equal(pos.long(), want_pos)
        want_slot = pt[b, want_pos // 16].long() * 16 + want_pos % 16
        assert torch.equal(slot, want_slot)
        hr = E[want_ids].float()
        torch.testing.assert_close(h, hr)
        xr = nw.float() * (hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + cfg.rms_eps))
        torch.testing.assert_close(x.float(), xr, rtol=1e-2, atol=1e-4)
    y = torch.randn((M, H), generator=g).to(DEV)
    wa, wb = _rand((H,), g, 0.02), _rand((H,), g, 0.02)
    h2 = torch.zeros_like(h)
    L.residual_norm(M, h, y, wa, wb, cfg.rms_eps, h2, x)
    torch.cuda.synchronize()
    rms = lambda t, w: w.float() * (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + cfg.rms_eps))
    hr2 = h + rms(y, wa)
    torch.testing.assert_close(h2, hr2, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(x.float(), rms(hr2, wb), rtol=1e-2, atol=1e-4)


# ---------------------------------------------------------------------- accept / commit (bit-exact)
def test_accept_commit_matches_reference_kernel_golden(golden_dir):
    """The reference Triton _ss_commit_kernel's own outputs (Triton CPU interpreter) on the same inputs."""
    data = json.load(open(os.path.join(golden_dir, "commit_kernel.json")))
    for case in data["cases"]:
        K, bs = case["K"], case["bs"]
        inp, want = case["in"], case["out"]
        pred = np.array(inp["predict"], dtype=np.int64)
        acc = inp["acc"]
        v = pred[: bs * K].reshape(bs, K)
        am = np.zeros((bs, K), dtype=np.int64)
        for i in range(bs):
            am[i, 0] = inp["a0"][i]
            for j in range(acc[i]):
                am[i, j + 1] = v[i, j]
            if acc[i] + 1 < K:
                am[i, acc[i] + 1] = v[i, acc[i]] + 1
            for j in range(acc[i] + 2, K):
                am[i, j] = v[i, j - 1]  # whatever follows a rejection cannot matter
        t32 = lambda a: torch.tensor(np.asarray(a), dtype=torch.int32, device=DEV)
        t64 = lambda a: torch.tensor(np.asarray(a), dtype=torch.int64, device=DEV)
        seeds, sl, loc = t64(inp["seeds"]), t64(inp["seq_lens"]), t64(inp["loc"])
        packed = torch.zeros((bs, K + 2), dtype=torch.int32, device=DEV)
        rel = torch.full((bs * K,), -1, dtype=torch.int64, device=DEV)
        nrel = torch.zeros((1,), dtype=torch.int32, device=DEV)
        out = torch.zeros((bs,), dtype=torch.int64, device=DEV)
        acc_d = torch.zeros((bs,), dtype=torch.int32, device=DEV)
        L.accept_commit(bs, K, t32(am.reshape(-1)), t32(v.reshape(-1)), seeds, t64(inp["rpi"]), sl, packed, rel, out,
                        x0_committed=True, loc=loc, n_released=nrel, accept_len=acc_d)
        torch.cuda.synchronize()
        assert acc_d.tolist() == acc
        assert packed.tolist() == want["packed"]
        assert seeds.tolist() == want["seeds"]
        assert sl.tolist() == want["seq_lens"]
        n = int(nrel.item())
        assert n == len(want["free"])
        assert rel[:n].tolist() == want["free"]
        assert out.tolist() == want["out"]


def test_accept_commit_random_vs_oracle():
    from oracle.commit_ref import batch_accept, released_positions
    rng = np.random.default_rng(7)
    for bs, K in [(1, 17), (64, 17), (300, 9), (128, 33), (7, 5)]:
        v = rng.integers(0, 59392, (bs, K))
        am = rng.integers(0, 59392, (bs, K))
        for i in range(bs):  # plant accepted prefixes of every length, full accept included
            a = rng.integers(0, K)
            am[i, 1: a + 1] = v[i, :a]
        acc = batch_accept(am, v)
        seq = rng.integers(100, 9000, bs)
        t = lambda a, dt: torch.tensor(np.asarray(a), dtype=dt, device=DEV)
        seeds = torch.zeros((bs + 3,), dtype=torch.int64, device=DEV)
        rpi = t(rng.permutation(bs + 3)[:bs], torch.int64)
        sl = t(seq, torch.int64)
        packed = torch.zeros((bs, K + 2), dtype=torch.int32, device=DEV)
        rel = torch.zeros((bs * K,), dtype=torch.int64, device=DEV)
        nrel = torch.zeros((1,), dtype=torch.int32, device=DEV)
        out = torch.zeros((bs,), dtype=torch.int64, device=DEV)
        ncom = torch.ones((bs,), dtype=torch.int32, device=DEV)
        rounds = torch.zeros((bs,), dtype=torch.int32, device=DEV)
        L.accept_commit(bs, K, t(am.reshape(-1), torch.int32), t(v.reshape(-1), torch.int32), seeds, rpi, sl, packed,
                        rel, out, x0_committed=False, n_released=nrel, n_committed=ncom, rounds=rounds)
        torch.cuda.synchronize()
        want_rel = [p for i in range(bs) for p in released_positions(int(seq[i]), int(acc[i]), K)]
        assert int(nrel.item()) == len(want_rel)
        assert rel[: len(want_rel)].tolist() == want_rel
        assert sl.tolist() == [int(seq[i] + acc[i] + 2) for i in range(bs)]
        assert out.tolist() == [int(v[i, acc[i]]) for i in range(bs)]
        assert ncom.tolist() == [int(1 + acc[i] + 2) for i in range(bs)]
        pk = packed.cpu().numpy()
        for i in range(bs):
            a = int(acc[i])
            assert pk[i, 0] == am[i, 0] and pk[i, 1] == a
            assert list(pk[i, 2: 3 + a]) == list(v[i, : a + 1]) and not pk[i, 3 + a:].any()


def test_draft_override_vs_oracle():
    from oracle.decoder_ref import forced_draft
    rng = np.random.default_rng(3)
    bs, K, V, mask_id = 5, 17, 59392, 59282
    glen = 200
    gs = rng.integers(0, V, (bs, glen))
    gs[0, 10] = mask_id - 1  # exercises the mask-id skip
    am = rng.integers(0, V, (bs, K))
    ncom = rng.integers(1, 100, bs)
    plan = rng.integers(0, K, (bs, 4))
    plan[:, 0] = [0, K - 1, K - 2, 3, 9]
    rounds = np.zeros(bs, dtype=np.int64)
    t = lambda a: torch.tensor(np.asarray(a), dtype=torch.int32, device=DEV)
    amd = t(am.reshape(-1))
    ncom[0] = 10 - (plan[0, 0] + 1)
    L.draft_override(bs, K, amd, t(gs), t(ncom), t(plan), t(rounds), V, mask_id)
    torch.cuda.synchronize()
    got = amd.view(bs, K).cpu()
    for b in range(bs):
        want = forced_draft(torch.tensor(am[b]), gs[b].tolist(), int(ncom[b]), int(plan[b, 0]), V, mask_id)
        assert got[b].tolist() == want.tolist()


def test_shared_workspace_across_shapes():
    """One scratch buffer serves every projection and lm_head of a forward, in any order and at any M (a shape's
    partial sums must never land on another shape's tickets)."""
    g = torch.Generator().manual_seed(41)
    shapes = [(4096, 1536, 17), (59392, 1536, 64), (1536, 2048, 17), (9216, 1536, 64), (1536, 4608, 17),
              (59392, 1536, 17), (4096, 1536, 64), (59392, 1536, 64)]
    need = max(L.linear_workspace_bytes(n, m, L.linear_default_splits(n, k, m, md)) for n, k, m in shapes
               for md in (L.EPI_STORE_F32, L.EPI_PARTIAL_F32))
    ws = torch.zeros((need,), dtype=torch.uint8, device=DEV)
    for n_out, k_in, m in shapes:
        w, x = _rand((n_out, k_in), g, 0.02), _rand((m, k_in), g)
        ref = x.float() @ w.float().T
        e = L.Epilogue()
        if n_out == 59392:
            idx = torch.full((m,), -1, dtype=torch.int32, device=DEV)
            top = torch.zeros((m,), device=DEV)
            e.mode, e.out_idx, e.out_top1 = L.EPI_ARGMAX, idx.data_ptr(), top.data_ptr()
            L.linear(w, x, m, e, ws)
            torch.cuda.synchronize()
            t2 = torch.topk(ref, 2, dim=-1)
            sure = (t2.values[:, 0] - t2.values[:, 1]) > 1e-3
            assert torch.equal(idx.long()[sure], t2.indices[:, 0][sure]), (n_out, k_in, m)
            torch.testing.assert_close(top, t2.values[:, 0], rtol=1e-4, atol=1e-3)
        else:
            out = torch.zeros((m, n_out), device=DEV)
            e.mode, e.out, e.ld_out = L.EPI_STORE_F32, out.data_ptr(), n_out
            L.linear(w, x, m, e, ws)
            torch.cuda.synchronize()
            torch.testing.assert_close(out, ref, rtol=1e-3, atol=2e-4 * math.sqrt(k_in))


def test_attention_shared_workspace_across_batches():
    nq, nkv, D, ps = 16, 8, 128, 16
    g = torch.Generator().manual_seed(9)
    n_pages = 900
    kc, vc = _rand((n_pages, nkv, ps, D), g), _rand((n_pages, nkv, ps, D), g)
    ws = torch.zeros((L.attention_workspace_bytes(64, 64, nq, nkv, 16),), dtype=torch.uint8, device=DEV)
    for bs, K, draft, chunk in [(1, 64, False, 128), (8, 17, True, 128), (1, 17, False, 256), (6, 33, True, 128)]:
        S = torch.randint(0, 1500, (bs,), generator=g)
        base_add = 0 if draft else 1
        P = (1600 + K) // ps + 2
        pt = torch.randint(0, n_pages, (bs, P), generator=g, dtype=torch.int32)
        q = _rand((bs * K, nq, D), g)
        pt_d, seq_d = pt.to(DEV), S.to(DEV)
        ms = int(math.ceil((int(S.max()) + base_add + K) / chunk))
        out = torch.zeros((bs * K, nq, D), dtype=torch.bfloat16, device=DEV)
        L.bd_attention(q, kc, vc, pt_d, seq_d, bs, K, draft, base_add, nq, nkv, ps, chunk, ms, out, ws)
        torch.cuda.synchronize()
        ref = _attn_ref(q, kc, vc, pt_d, seq_d, K, draft, base_add, nq, nkv)
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=1.5e-2)


@pytest.mark.parametrize("n_out,k_in,m", [(1536, 2048, 17), (1536, 4608, 17), (1536, 4608, 1088), (1536, 2048, 300),
                                          (1024, 2048, 33), (2048, 1024, 129)])
def test_linear_partials_summed_by_residual_norm(n_out, k_in, m):
    """o_proj / down_proj write split-K partials; the residual norm sums them in split order."""
    g = torch.Generator().manual_seed(m + k_in)
    w, x = _rand((n_out, k_in), g, 0.02), _rand((m, k_in), g)
    sp = L.linear_default_splits(n_out, k_in, m, L.EPI_PARTIAL_F32)
    y = torch.full((sp, m, n_out), float("nan"), device=DEV)
    e = L.Epilogue()
    e.mode, e.out, e.ld_out = L.EPI_PARTIAL_F32, y.data_ptr(), n_out
    L.linear(w, x, m, e, _ws(n_out, k_in, m, 1), splits=sp)
    h = torch.randn((m, n_out), generator=g).to(DEV) * 0.1
    wa, wb = _rand((n_out,), g, 0.02), _rand((n_out,), g, 0.02)
    h2 = torch.zeros_like(h)
    xo = torch.zeros((m, n_out), dtype=torch.bfloat16, device=DEV)
    L.residual_norm(m, h, y, wa, wb, 1e-5, h2, xo, y_parts=sp)
    torch.cuda.synchronize()
    ref_y = x.float() @ w.float().T
    torch.testing.assert_close(y.sum(0), ref_y, rtol=1e-3, atol=2e-4 * math.sqrt(k_in))
    rms = lambda t, ww: ww.float() * (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-5))
    hr = h + rms(ref_y, wa)
    torch.testing.assert_close(h2, hr, rtol=1e-3, atol=1e-5)
    torch.testing.assert_close(xo.float(), rms(hr, wb), rtol=1e-2, atol=1e-4)


@pytest.mark.parametrize("parts", [1, 2, 3, 4, 5])
def test_residual_norm_many_rows_kernel(parts):
    """Above 512 rows the norm runs a fixed grid of CTAs that walk the rows with the next row's loads in flight (up to
    four partials; five fall back to one CTA per row).  Against the fp32 reference, and bit for bit against the
    few-rows kernel on the rows both calls compute (same arithmetic in the same order)."""
    m, H = 1088, 1536
    g = torch.Generator().manual_seed(parts)
    y = torch.randn((parts, m, H), generator=g).to(DEV) * 0.3
    h = torch.randn((m, H), generator=g).to(DEV) * 0.1
    wa, wb = _rand((H,), g, 0.02), _rand((H,), g, 0.02)
    h2 = torch.full_like(h, float("nan"))
    xo = torch.zeros((m, H), dtype=torch.bfloat16, device=DEV)
    L.residual_norm(m, h, y, wa, wb, 1e-5, h2, xo, y_parts=parts)
    few = 500
    yf = y[:, :few].contiguous()
    h2f = torch.full((few, H), float("nan"), device=DEV)
    xof = torch.zeros((few, H), dtype=torch.bfloat16, device=DEV)
    L.residual_norm(few, h[:few].contiguous(), yf, wa, wb, 1e-5, h2f, xof, y_parts=parts)
    torch.cuda.synchronize()
    rms = lambda t, ww: ww.float() * (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-5))
    hr = h + rms(y.sum(0), wa)
    torch.testing.assert_close(h2, hr, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(xo.float(), rms(hr, wb), rtol=1e-2, atol=1e-4)
    assert torch.equal(h2[:few], h2f) and torch.equal(xo[:few], xof)


@pytest.mark.parametrize("bs,K,draft,chunk,q_scale", [(64, 17, False, 4096, 1.0), (64, 17, True, 4096, 1.0),
                                                     (24, 17, False, 512, 1.0), (24, 17, True, 256, 4.0),
                                                     (40, 9, False, 1024, 8.0), (20, 32, True, 4096, 1.0),
                                                     (12, 33, True, 1024, 1.0), (20, 64, False, 4096, 2.0),
                                                     (1, 17, False, 256, 1.0), (2, 17, True, 512, 4.0),
                                                     (1, 17, True, 192, 1.0), (4, 33, False, 4096, 1.0),
                                                     (3, 17, False, 1024, 8.0), (40, 17, False, 2560, 1.0)])
def test_attention_tc_matches_mma_kernel(bs, K, draft, chunk, q_scale):
    """The tcgen05 / TMEM kernel against the fp32 reference and the mma.sync kernel on the same inputs: large grids
    (more units than SMs; global split merge) and small grids (one CTA per SM; the splits of a (request, kv head) as
    one cluster merging through distributed shared memory).  Scaled queries make the reference max move often (the O
    rescale in TMEM); small chunks give split partials and the merges.  Prefixes U[0, 3000] (seed 11)."""
    nq, nkv, D, ps = 16, 8, 128, 16
    g = torch.Generator().manual_seed(11)
    S = torch.randint(0, 3001, (bs,), generator=g)
    base_add = 0 if draft else 1
    need = [(int(s) + base_add + K + ps - 1) // ps for s in S]
    P = max(need) + 1
    n_pages = sum(need) + 4
    perm = torch.randperm(n_pages, generator=g)
    pt = torch.zeros((bs, P), dtype=torch.int32)
    o = 0
    for b in range(bs):
        pt[b, : need[b]] = perm[o: o + need[b]].to(torch.int32)
        pt[b, need[b]:] = perm[o]
        o += need[b]
    kc = _rand((n_pages, nkv, ps, D), g)
    vc = _rand((n_pages, nkv, ps, D), g)
    q = _rand((bs * K, nq, D), g, scale=q_scale)
    pt_d, seq_d = pt.to(DEV), S.to(DEV)
    Lmax = int(S.max()) + base_add + K
    max_splits = int(math.ceil(Lmax / chunk))
    assert max_splits <= 16
    ws = torch.zeros((L.attention_workspace_bytes(bs, K, nq, nkv, max_splits),), dtype=torch.uint8, device=DEV)
    st = torch.zeros((1,), dtype=torch.int32, device=DEV)
    outs = []
    try:
        for tc in (2, 0):
            L.set_attention_tc(tc)
            out = torch.full((bs * K, nq, D), float("nan"), dtype=torch.bfloat16, device=DEV)
            L.bd_attention(q, kc, vc, pt_d, seq_d, bs, K, draft, base_add, nq, nkv, ps, chunk, max_splits, out, ws,
                           status=st)
            torch.cuda.synchronize()
            assert int(st.item()) == 0
            outs.append(out.float())
    finally:
        L.set_attention_tc(True)
    ref = _attn_ref(q, kc, vc, pt_d, seq_d, K, draft, base_add, nq, nkv)
    torch.testing.assert_close(outs[0], ref, rtol=2e-2, atol=1.5e-2)
    torch.testing.assert_close(outs[0], outs[1], rtol=2e-2, atol=1.5e-2)
