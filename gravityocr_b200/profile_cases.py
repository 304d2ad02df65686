"""Small, self-contained launches of one kernel for ncu captures (a few GB on the device at most, inputs larger than
L2, a handful of launches).  Example:

    python -m gravityocr_b200.profile_cases attention --bs 16 --seq 2048 --reps 3
    ncu --set full --clock-control none -k regex:attention_kernel -s 1 -c 2 \\
        python -m gravityocr_b200.profile_cases attention --bs 16 --seq 2048 --reps 3

Every case first runs one untimed warm-up launch, then ``--reps`` launches, and prints the mean CUDA-event time and
the algorithmic bytes / FLOPs of one launch.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from . import _lib as L
from .config import ModelConfig
from .engine import rope_inv_freq
from .metrics import attention_bytes


GRAPH = False  # --graph: time `reps` launches captured in one CUDA graph (device-bound, as in the engine)


def _time(fn, reps):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if GRAPH:
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def case_attention(a):
    cfg = ModelConfig()
    bs, K = a.bs, a.bd + 1
    g = torch.Generator().manual_seed(1)
    nq, nkv, D, ps = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, 16
    if a.mixed:
        # the config-3 mix: prefixes U[256, 4096] image tokens + 32 prompt tokens (seed 3)
        S = (torch.randint(256, 4097, (bs,), generator=torch.Generator().manual_seed(3)) + 32).tolist()
    else:
        S = [a.seq] * bs
    seq_max = max(S)
    ppr = (seq_max + K + 2 + ps - 1) // ps
    n_pages = bs * ppr
    kc = torch.randn((n_pages, nkv, ps, D), generator=g).to("cuda", torch.bfloat16)
    vc = torch.randn((n_pages, nkv, ps, D), generator=g).to("cuda", torch.bfloat16)
    pt = torch.randperm(n_pages, generator=g).to(torch.int32).view(bs, ppr).cuda()
    seq = torch.tensor(S, dtype=torch.int64, device="cuda")
    avg = sum(S) // len(S)
    q = torch.randn((bs * K, nq, D), generator=g).to("cuda", torch.bfloat16)
    out = torch.empty_like(q)
    from .engine import attention_split
    chunk, splits = attention_split(bs, K, seq_max, avg, nkv, L.num_sms())
    if a.chunk:
        chunk, splits = a.chunk, int(math.ceil((seq_max + K + 1) / a.chunk))
    ws = torch.zeros((L.attention_workspace_bytes(bs, K, nq, nkv, splits),), dtype=torch.uint8, device="cuda")
    order = torch.argsort(seq, descending=True, stable=True).to(torch.int32) if a.mixed else None
    fn = lambda: L.bd_attention(q, kc, vc, pt, seq, bs, K, a.draft, 0 if a.draft else 1, nq, nkv, ps, chunk, splits,
                                out, ws, order=order)
    L.set_attention_tc(0 if a.mma else (2 if a.tc_all else 1))
    ms = _time(fn, a.reps)
    b = attention_bytes(cfg, S, K, 0 if a.draft else 1)
    tc = not a.mma and nq // nkv * K <= 128 and (a.tc_all or bs * nkv * splits > L.num_sms())
    return {"kernel": "attention_tc_kernel" if tc else "attention_kernel", "bs": bs, "seq": "mixed" if a.mixed else a.seq, "K": K, "chunk": chunk,
            "splits": splits, "ms": ms,
            "bytes": b, "GBps": b / ms / 1e6}


def case_linear(a):
    cfg = ModelConfig()
    n_out, k_in, m = a.n_out, a.k_in, a.m
    g = torch.Generator().manual_seed(2)
    w = (torch.randn((n_out, k_in), generator=g) * 0.02).to("cuda", torch.bfloat16)
    x = torch.randn((m, k_in), generator=g).to("cuda", torch.bfloat16)
    mode = {"f32": L.EPI_STORE_F32, "partial": L.EPI_PARTIAL_F32, "swiglu": L.EPI_SWIGLU, "argmax": L.EPI_ARGMAX,
            "qkv": L.EPI_QKV_ROPE}[a.epi]
    sp = a.splits or L.linear_default_splits(n_out, k_in, m)
    e = L.Epilogue()
    e.mode = mode
    keep = []
    if mode in (L.EPI_STORE_F32, L.EPI_PARTIAL_F32):
        out = torch.zeros(((sp if mode == L.EPI_PARTIAL_F32 else 1) * m, n_out), device="cuda")
        e.out, e.ld_out = out.data_ptr(), n_out
        keep.append(out)
    elif mode == L.EPI_SWIGLU:
        out = torch.zeros((m, n_out // 2), dtype=torch.bfloat16, device="cuda")
        e.out, e.ld_out = out.data_ptr(), n_out // 2
        keep.append(out)
    elif mode == L.EPI_ARGMAX:
        idx = torch.zeros((m,), dtype=torch.int32, device="cuda")
        e.out_idx = idx.data_ptr()
        keep.append(idx)
    else:
        q = torch.zeros((m, cfg.q_dim), dtype=torch.bfloat16, device="cuda")
        kc = torch.zeros((m // 16 + 2, cfg.n_kv_heads, 16, 128), dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        pos = torch.arange(m, dtype=torch.int32, device="cuda")
        slot = torch.arange(m, dtype=torch.int64, device="cuda")
        inv = rope_inv_freq(cfg).cuda()
        e.q_out, e.k_cache, e.v_cache = q.data_ptr(), kc.data_ptr(), vc.data_ptr()
        e.row_pos, e.row_slot, e.inv_freq = pos.data_ptr(), slot.data_ptr(), inv.data_ptr()
        e.rotary_dim, e.n_q_heads, e.n_kv_heads, e.page_size = cfg.rotary_dim, cfg.n_q_heads, cfg.n_kv_heads, 16
        keep += [q, kc, vc, pos, slot, inv]
    ws_sp = 1 if mode == L.EPI_PARTIAL_F32 else sp
    ws = torch.zeros((L.linear_workspace_bytes(n_out, m, ws_sp),), dtype=torch.uint8, device="cuda")
    ms = _time(lambda: L.linear(w, x, m, e, ws, splits=sp), a.reps)
    wb = n_out * k_in * 2
    fl = 2 * n_out * k_in * m
    return {"kernel": "linear_kernel", "epi": a.epi, "n_out": n_out, "k_in": k_in, "m": m, "splits": sp, "ms": ms,
            "weight_GBps": wb / ms / 1e6, "TFLOPs": fl / ms / 1e9}


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="case", required=True)
    at = sub.add_parser("attention")
    at.add_argument("--bs", type=int, default=16)
    at.add_argument("--seq", type=int, default=2048)
    at.add_argument("--bd", type=int, default=16)
    at.add_argument("--draft", action="store_true")
    at.add_argument("--chunk", type=int, default=0)
    at.add_argument("--mixed", action="store_true", help="config-3 prefix lengths instead of --seq")
    at.add_argument("--mma", action="store_true", help="every grid on the mma.sync kernel")
    at.add_argument("--tc-all", action="store_true", help="every grid on the tcgen05 kernel (small grids included)")
    at.add_argument("--reps", type=int, default=3)
    li = sub.add_parser("linear")
    li.add_argument("--n-out", type=int, default=9216)
    li.add_argument("--k-in", type=int, default=1536)
    li.add_argument("--m", type=int, default=17)
    li.add_argument("--epi", default="swiglu", choices=["f32", "partial", "swiglu", "argmax", "qkv"])
    li.add_argument("--splits", type=int, default=0)
    li.add_argument("--reps", type=int, default=3)
    ap.add_argument("--graph", action="store_true", help="time launches captured in one CUDA graph")
    a = ap.parse_args()
    global GRAPH
    GRAPH = a.graph
    r = case_attention(a) if a.case == "attention" else case_linear(a)
    print(json.dumps(r))


if __name__ == "__main__":
    main()
