#!/usr/bin/env python
"""Benchmark of the self-speculative decode round on B200s (driver contract: one JSON line from rank 0).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one replica per GPU, requests sharded, no collective)

Workload (weak scaling): 64 concurrent requests per GPU, prefixes U[256, 4096] image-embedding
tokens + 32 prompt tokens, B = 16 (K = 17 rows per forward), paged K/V with 16-token pages, bf16, seed 3; random-init
weights N(0, 0.02) (no checkpoint), synthetic inputs (no dataset).  Prefill runs first (not timed).  A step is one
self-spec round over the whole batch: draft forward + causal verify forward + accept-and-commit, replayed from CUDA
graphs with every length, seed and page table resident on the device.  value = committed tokens of all ranks / the
slowest rank's device time.  The workload is far larger than L2 (1.16 GB of weights and ~11 GB of K/V per forward).

Also reported on rank 0 at N = 1: the bs-1 crop workload (config 2: prefix 256 + 32, 1024 tokens) in natural and
forced-accept replay modes, per-forward % of the measured HBM roofline, the dominant kernel's roofline, the
end-to-end number through the served worker API (per-round H2D of the batch's request slots and D2H of the packed
commit rows), and the CPU port of the reference round on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "self-spec decode tokens/s & tokens/forward @bs1/bs64, %HBM roofline, 1/2/4/8 B200"
K_BD = 16
SEED = 3
# DRAM bytes / algorithmic bytes of one verify attention launch (attention_tc_kernel) on the config-3 mix:
# dram__bytes_read.sum + dram__bytes_write.sum of an ncu capture of that launch over its algorithmic bytes
ATTN_TRAFFIC_RATIO = (584.55e6 + 5.84e6) / 586.94e6


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    # 20 rounds: the configuration every recorded figure uses (each round lengthens every request's K/V, so longer runs
    # measure longer sequences: 200 rounds ran 8.29 ms per round at 30.9K tokens/s on a box at 1,725 MHz)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--bd", type=int, default=K_BD)
    ap.add_argument("--no-bs1", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile-small", action="store_true", help="short run for ncu captures (no extras)")
    ap.add_argument("--config4", action="store_true",
                    help="config-4 sweep instead: prefix 4096 + 64, B in {4, 8, 16, 32}, batch 1 and 128")
    return ap.parse_args()


def peaks():
    """(HBM GB/s, dense bf16 TF/s burst, dense bf16 TF/s sustained, source)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def prefill_line(cfg, prefix, seconds, tc_sustained, peak_src, chunk):
    """The prefill before the timed rounds (wall clock, host input staging included), against the dense causal
    prefill's algorithmic FLOPs at the sustained bf16 peak."""
    from gravityocr_b200.metrics import prefill_flops
    fl = prefill_flops(cfg, prefix)
    return {"tokens": int(sum(prefix)), "s": round(seconds, 3), "tokens_per_s": round(sum(prefix) / seconds, 1),
            "tflops": round(fl / seconds / 1e12, 1), "tensor_frac": round(fl / seconds / 1e12 / tc_sustained, 4),
            "peak": f"{peak_src} bf16 GEMM sustained", "flops": fl,
            "how": f"chunks of {chunk} rows per request through the decode kernels (the attention kernel holds a "
                   f"request's {chunk} query rows in one tile); not in the timed region"}


def forward_bound(cfg, seqs, K, verify, ms, hbm_peak, tc_sustained):
    """A forward's time against its roofline.  hbm_frac / tensor_frac: all bytes / HBM peak and all FLOPs / sustained
    tensor peak over the forward's time.  serial_bound_frac: the forward runs its phases one after another, so its
    bound is the sum of the phases' bounds -- the attention launches at K/V bytes / HBM peak plus the projections
    (weights, lm_head included) at max(weight bytes / HBM peak, GEMM FLOPs / tensor peak)."""
    from gravityocr_b200.metrics import forward_bytes, forward_flops
    b = forward_bytes(cfg, seqs, K, verify)
    f = forward_flops(cfg, seqs, K, verify)
    t_hbm = b / (hbm_peak * 1e9)
    t_tc = f / (tc_sustained * 1e12)
    w_bytes = cfg.streamed_params() * 2
    gemm_flops = 2 * cfg.streamed_params() * len(seqs) * K
    t_attn = (b - w_bytes) / (hbm_peak * 1e9)
    t_gemm = max(w_bytes / (hbm_peak * 1e9), gemm_flops / (tc_sustained * 1e12))
    t = ms / 1e3
    return {"bytes": b, "flops": f, "hbm_frac": round(t_hbm / t, 4), "tensor_frac": round(t_tc / t, 4),
            "serial_bound_ms": round((t_attn + t_gemm) * 1e3, 4), "serial_bound_frac": round((t_attn + t_gemm) / t, 4),
            "gemm_bound": "tensor" if gemm_flops / (tc_sustained * 1e12) > w_bytes / (hbm_peak * 1e9) else "hbm",
            "ms": round(ms, 4)}


# ---------------------------------------------------------------------- workload
def workload(cfg, n_req: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    n_img = torch.randint(256, 4097, (n_req,), generator=g).tolist()
    out_len = torch.randint(256, 2049, (n_req,), generator=g).tolist()
    return n_img, out_len


def request_rows(cfg, weights, seed, idx, n_img, n_prompt=32):
    from gravityocr_b200.weights import request_inputs
    img, txt = request_inputs(cfg, seed, n_img, n_prompt, idx, torch.bfloat16)
    emb = weights["embed_tokens"][txt].float()
    x = torch.cat([img, emb], 0)
    ids = torch.cat([torch.full((n_img,), -1, dtype=torch.int64), txt])
    return x, ids


class ClockSampler:
    """nvidia-smi samples (200 ms) during the timed region."""

    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={','.join(self.FIELDS)}", "--format=csv,noheader,nounits",
                                       "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.p is not None:
            time.sleep(0.25)
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------- CPU port of the reference round
def cpu_round_port(cfg, weights, x, K, rounds, threads=None):
    """The oracle's restatement of the reference round (fp32 torch on the CPU, all host threads) on one request: a real
    causal prefill of its prefix rows x (not timed, as the reference's decode-loop timing excludes prefill), then
    `rounds` full-draft rounds, timed.  Returns (tokens/s, committed tokens, seconds, threads, tokens per forward)."""
    from oracle.decoder_ref import OracleDecoder, spec_round, spec_start
    n = threads or os.cpu_count() or 1
    torch.set_num_threads(n)
    m = OracleDecoder(cfg, weights)
    st = spec_start(m, x, x.shape[0] + rounds * (K + 1) + K + 2)
    t0 = time.perf_counter()
    for _ in range(rounds):
        spec_round(m, st, K)
    secs = time.perf_counter() - t0
    toks = len(st.out) - 1
    return toks / secs, toks, secs, n, toks / (2 * rounds)


def cpu_sample(cfg, w, idx, n_img):
    """The bounded CPU sample: the shortest request of the shard (its prefill stays within seconds)."""
    i = min(range(len(idx)), key=lambda k: (n_img[idx[k]], idx[k]))
    x, _ = request_rows(cfg, w, SEED, idx[i], n_img[idx[i]])
    return idx[i], x


def run_reference(a):
    from gravityocr_b200 import dp
    from gravityocr_b200.config import ModelConfig
    from gravityocr_b200.weights import random_weights
    rank, world, _ = dp.dist_env()
    if rank != 0:
        return 0
    cfg = ModelConfig()
    K = a.bd + 1
    w = random_weights(cfg, SEED, torch.bfloat16)
    w32 = {k: v.float() for k, v in w.items()}
    n_img, _ = workload(cfg, a.batch, SEED)
    ridx, x = cpu_sample(cfg, w, list(range(a.batch)), n_img)
    rounds = max(1, min(4, a.steps))
    tps, toks, secs, n, tpf = cpu_round_port(cfg, w32, x, K, rounds)
    steps_done = a.warmup + a.steps
    line = {"impl": "reference", "metric": METRIC, "value": round(tps, 4), "unit": "tokens/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(1000 * secs / rounds, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": f"config3-bs64-serving (CPU sample: request {ridx})", "batch_per_gpu": a.batch,
                       "K": K, "prefix": int(x.shape[0]), "page_size": 16},
            "tokens_per_forward": round(tpf, 4),
            "cpu_baseline": {"value": round(tps, 4), "unit": "tokens/s", "cores": n, "kind": "port",
                             "sample": f"{rounds} full-draft rounds of request {ridx} after its real prefill "
                                       f"({int(x.shape[0])} prefix tokens), fp32 torch on {n} host threads"},
            "e2e": {"value": round(tps, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's round is Python over SGLang / transformers and its source tree is not on the GPU "
                    "box, so the arm times the oracle's CPU restatement of that round (pinned to the reference's own "
                    "outputs in the test suite)", "steps_run": steps_done}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------- native
def time_graphs(gd, gv, steps):
    """Replay draft and verify graphs `steps` times; returns (total ms, draft ms, verify ms)."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for e in ev:
        e[0].record()
        gd.replay()
        e[1].record()
        gv.replay()
        e[2].record()
    t1.record()
    torch.cuda.synchronize()
    d = sum(e[0].elapsed_time(e[1]) for e in ev)
    v = sum(e[1].elapsed_time(e[2]) for e in ev)
    return t0.elapsed_time(t1), d, v


def main():
    a = _args()
    if a.impl == "reference":
        return run_reference(a)
    if a.config4:
        return config4_sweep(a)
    from gravityocr_b200 import _lib as L
    from gravityocr_b200 import dp
    from gravityocr_b200.config import ModelConfig
    from gravityocr_b200.engine import Engine
    from gravityocr_b200.metrics import attention_bytes, forward_bytes
    from gravityocr_b200.weights import random_weights

    rank, world, local = dp.dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dp.init("nccl" if world > 1 else "gloo", timeout_s=600)
    hbm_peak, tc_peak, tc_sus, peak_src = peaks()
    cfg = ModelConfig()
    K = a.bd + 1
    bs = a.batch
    w = random_weights(cfg, SEED, torch.bfloat16)

    # ---- this rank's requests: equal-count, work-balanced shard of the global request list
    n_img, out_len = workload(cfg, bs * world, SEED)
    work = [n_img[i] + 32 + out_len[i] for i in range(bs * world)]
    mine = dp.balanced_shards(work, world)[rank]
    prefix = [n_img[i] + 32 for i in mine]
    rounds_max = a.warmup + a.steps + 8   # the end-to-end run rewinds to the pre-warm-up state and replays the same rounds
    cap = max(prefix) + rounds_max * (K + 1) + 2 * K + 64
    ppr = (cap + 15) // 16
    chunk = 64
    eng = Engine(cfg, w, max_rows=max(bs * K, bs * chunk), n_pages=bs * ppr + 8 + 256, device=dev)  # +256: bs-1 run
    eng.reserve(bs * K)
    rb = eng.new_round_buffers(bs, K, ppr, max_len=cap, avg_len=int(sum(prefix) / len(prefix)))
    for b in range(bs):
        rb.page_table[b] = torch.tensor(eng.pool.alloc(ppr), dtype=torch.int32, device=dev)
    xs, ids = zip(*[request_rows(cfg, w, SEED, i, n_img[i]) for i in mine])
    t_pf = time.perf_counter()
    eng.prefill(rb, list(xs), list(ids), chunk=chunk)
    torch.cuda.synchronize()
    t_pf = time.perf_counter() - t_pf
    del xs, ids

    # ---- graphs (one eager round first: sizes every scratch buffer before capture)
    eng.round_launch(rb)
    torch.cuda.synchronize()
    eng.check_status(rb)
    gd, gv = eng.capture_split(rb)
    # round state before the warm-up: the end-to-end run replays the same warm-up and timed rounds from here
    state0 = (rb.seq_lens.clone(), rb.seeds.clone(), rb.n_committed.clone(), rb.rounds.clone())
    for _ in range(a.warmup):
        gd.replay()
        gv.replay()
    torch.cuda.synchronize()
    eng.check_status(rb)

    ncom0 = rb.n_committed.clone()
    seq0 = rb.seq_lens.cpu().tolist()
    dp.barrier(dev)
    torch.cuda.synchronize()
    prof = os.environ.get("GR_PROFILE_RANGE") == "1"  # ncu --profile-from-start off: capture the timed rounds only
    with ClockSampler(local) as clk:
        if prof:
            torch.cuda.cudart().cudaProfilerStart()
        total_ms, draft_ms, verify_ms = time_graphs(gd, gv, a.steps)
        if prof:
            torch.cuda.cudart().cudaProfilerStop()
    dp.barrier(dev)
    eng.check_status(rb)
    seq1 = rb.seq_lens.cpu().tolist()
    tokens = int((rb.n_committed - ncom0).sum().item())
    final_dev = (rb.seq_lens.cpu().tolist(), rb.seeds.cpu().tolist(), (rb.n_committed - state0[2]).cpu().tolist())
    elapsed = dp.max_over_ranks(total_ms, dev)
    tokens_all = dp.sum_over_ranks(float(tokens), dev)
    value = tokens_all / (elapsed / 1000.0)
    fwd = 2 * a.steps
    tok_per_fwd = tokens / (fwd * bs)
    # per-forward rooflines (average over the timed rounds: the lengths grow linearly)
    seq_mid = [(x + y) / 2 for x, y in zip(seq0, seq1)]
    bd = forward_bytes(cfg, seq_mid, K, verify=False)
    bv = forward_bytes(cfg, seq_mid, K, verify=True)
    frac_d = bd / (draft_ms / a.steps / 1000.0) / (hbm_peak * 1e9)
    frac_v = bv / (verify_ms / a.steps / 1000.0) / (hbm_peak * 1e9)
    bound_d = forward_bound(cfg, seq_mid, K, False, draft_ms / a.steps, hbm_peak, tc_sus)
    bound_v = forward_bound(cfg, seq_mid, K, True, verify_ms / a.steps, hbm_peak, tc_sus)
    # work-normalised throughput: forward rows (bs x K per forward) per second, independent of how many drafts a
    # shard's requests happen to accept
    rows_s = dp.sum_over_ranks(float(2 * a.steps * bs * K), dev) / (elapsed / 1000.0)
    per_rank = dp.gather_objects({"rank": rank, "tokens": tokens, "tokens_per_forward": round(tok_per_fwd, 4),
                                  "ms_per_step": round(total_ms / a.steps, 4)})

    # ---- dominant kernel at this batch: the verify attention (K/V streaming); timed alone on this stream
    seq_now = rb.seq_lens.cpu().tolist()
    ws = eng._attn_workspace(bs, K, rb.attn_splits)
    st = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_rep = 20
    for i in range(n_rep + 3):
        if i == 3:
            ev0.record(st)
        l = i % cfg.n_layers  # rotate layers: each launch reads K/V that is not in L2
        L.bd_attention(eng.q, eng.pool.k[l], eng.pool.v[l], rb.page_table, rb.seq_lens, bs, K, False, 1,
                       cfg.n_q_heads, cfg.n_kv_heads, 16, rb.attn_chunk, rb.attn_splits, eng.attn, ws, status=rb.status,
                       order=rb.order)
    ev1.record(st)
    torch.cuda.synchronize()
    attn_ms = ev0.elapsed_time(ev1) / n_rep
    attn_b = attention_bytes(cfg, seq_now, K, 1)
    attn_gbs = attn_b / (attn_ms / 1000.0) / 1e9
    launches = a.steps * (2 * eng.kernels_per_forward(bs * K) + 1)

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(elapsed / a.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights N(0,0.02) and inputs; no checkpoint or dataset)",
        "config": {"workload": "config3-bs64-serving", "batch_per_gpu": bs, "bd_size": a.bd, "K": K, "page_size": 16,
                   "prefix": "U[256,4096] image + 32 prompt", "seed": SEED, "parallelism": f"dp{world} (replicas)",
                   "l2": "inputs larger than L2 (1.16 GB weights + K/V per forward)",
                   "no_finish": "output budgets U[256,2048] exceed the timed rounds"},
        "tokens_per_forward": round(tok_per_fwd, 4),
        "rows_per_s": round(rows_s, 1),
        "per_rank": per_rank,
        "hbm_roofline_per_forward": {"draft": round(frac_d, 4), "verify": round(frac_v, 4), "peak_gbs": hbm_peak,
                                     "peak": peak_src, "draft_ms": round(draft_ms / a.steps, 4),
                                     "verify_ms": round(verify_ms / a.steps, 4),
                                     "bytes_draft": bd, "bytes_verify": bv},
        "bound_per_forward": {"draft": bound_d, "verify": bound_v, "hbm_gbs": hbm_peak, "tensor_tflops": tc_sus,
                              "peak": f"{peak_src} (HBM copy; bf16 GEMM sustained)"},
        "roofline": {"kernel": "attention_tc_kernel (verify, one layer)", "bound": "hbm",
                     "achieved": round(attn_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(attn_gbs / hbm_peak, 4), "traffic": int(attn_b * ATTN_TRAFFIC_RATIO),
                     "traffic_source": "ncu dram bytes of the same kernel on the config-3 mix, scaled to this launch",
                     "algorithmic_bytes": attn_b, "avg_launch_ms": round(attn_ms, 5), "peak_source": peak_src},
        "gpu_launches": launches,
        "prefill_s": round(t_pf, 2),
        "prefill": prefill_line(cfg, prefix, t_pf, tc_sus, peak_src, chunk),
    }
    if rank == 0:
        line["clocks"] = clk.summary()

    # ---- end to end through the served worker API: the same warm-up and timed rounds as the device-timed run,
    # replayed from the saved round state (the rounds are deterministic, so they rewrite the same K/V rows and must
    # commit the same tokens)
    if not a.no_e2e and not a.profile_small:
        for t, t0 in zip((rb.seq_lens, rb.seeds, rb.n_committed, rb.rounds), state0):
            t.copy_(t0)
        e2e = e2e_worker(eng, rb, cfg, K, a.steps, dev, a.warmup)
        final_e2e = e2e.pop("final")
        same = final_e2e == final_dev and e2e["tokens"] == tokens
        if not same:
            raise RuntimeError("the end-to-end rounds did not commit what the device-timed rounds committed")
        tok_all = dp.sum_over_ranks(float(e2e.pop("tokens")), dev)
        ms_max = dp.max_over_ranks(e2e.pop("ms"), dev)
        e2e["value"] = round(tok_all / (ms_max / 1000.0), 2)
        e2e["same_tokens_as_device_run"] = same
        line["e2e"] = e2e

    if rank == 0 and world == 1 and not a.profile_small:
        line["draining_batch_attention"] = draining_attention(eng, rb, cfg, K, hbm_peak)
        line["sampled"] = sampled_rounds(eng, rb, cfg, K, min(a.steps, 10), dev)
        if not a.no_bs1:
            line["bs1"] = bs1_crop(eng, cfg, w, K, dev, hbm_peak)
        if not a.no_cpu:
            w32 = {k: v.float() for k, v in w.items()}
            ridx, x = cpu_sample(cfg, w, mine, n_img)
            tps, toks, secs, n, tpf = cpu_round_port(cfg, w32, x, K, 4)
            line["cpu_baseline"] = {"value": round(tps, 4), "unit": "tokens/s", "cores": n, "kind": "port",
                                    "tokens_per_forward": round(tpf, 4),
                                    "sample": f"4 full-draft rounds of config-3 request {ridx} after its real prefill "
                                              f"({int(x.shape[0])} prefix tokens), fp32 torch on {n} host threads: "
                                              f"{toks} tokens in {secs:.1f} s"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    dp.finish()
    return 0


def draining_attention(eng, rb, cfg, K, hbm_peak):
    """The verify attention of a batch that drains as requests finish: the first bs requests of the workload (their
    real K/V in the cache, config-3 prefixes) at bs 8, 16 and 32 with the engine's split plan; one layer per launch,
    rotating layers so each launch reads K/V that is not in L2."""
    from gravityocr_b200 import _lib as L
    from gravityocr_b200.engine import attention_split
    from gravityocr_b200.metrics import attention_bytes
    out = {}
    for bs in (8, 16, 32):
        seq = rb.seq_lens[:bs].contiguous()
        pt = rb.page_table[:bs].contiguous()
        S = seq.cpu().tolist()
        order = torch.argsort(seq, descending=True, stable=True).to(torch.int32)
        chunk, splits = attention_split(bs, K, max(S), int(sum(S) / bs), cfg.n_kv_heads, eng.sms)
        ws = torch.zeros((L.attention_workspace_bytes(bs, K, cfg.n_q_heads, cfg.n_kv_heads, splits),),
                         dtype=torch.uint8, device=eng.device)
        q = eng.q[: bs * K]
        o = eng.attn[: bs * K]
        def launch(l):
            L.bd_attention(q, eng.pool.k[l], eng.pool.v[l], pt, seq, bs, K, False, 1, cfg.n_q_heads, cfg.n_kv_heads,
                           16, chunk, splits, o, ws, status=rb.status, order=order)
        for i in range(3):
            launch(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(32):
            launch(i % cfg.n_layers)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / 32 * 1000
        b = attention_bytes(cfg, S, K, 1)
        out[f"bs{bs}"] = {"us": round(us, 2), "chunk": chunk, "splits": splits, "gbs": round(b / us / 1e3, 1),
                          "hbm_frac": round(b / us / 1e3 / hbm_peak, 4)}
    eng.check_status(rb)
    return out


def sampled_rounds(eng, rb, cfg, K, steps, dev):
    """The same batch as a non-plain batch (temperature 0.8, top-p 0.95, top-k 50, repetition 1.1, frequency 0.1):
    draft, a0 draw, verify, speculative sampling of the verify rows, commit, penalizer cumulation -- device time per
    round against the greedy round's (eager launches, not graphs, on both sides of the comparison)."""
    from gravityocr_b200.sampling import RequestSampling, SampledRound, SamplerState
    bs = rb.bs
    st = SamplerState(cfg.vocab, rb.seeds.shape[0], dev, seed=SEED)
    rs = [RequestSampling(temperature=0.8, top_p=0.95, top_k=50, repetition_penalty=1.1, frequency_penalty=0.1)] * bs
    smp = st.batch(rs, rb.rpi)
    sr = SampledRound(eng, rb)
    snap = (rb.seq_lens.clone(), rb.seeds.clone(), rb.n_committed.clone(), rb.rounds.clone())

    def restore():
        for t, t0 in zip((rb.seq_lens, rb.seeds, rb.n_committed, rb.rounds), snap):
            t.copy_(t0)

    out = {}
    for name in ("greedy", "sampled"):
        restore()
        for _ in range(2):
            if name == "greedy":
                eng.round_launch(rb)
            else:
                sr.draft(smp)
                sr.verify(smp, st.rng)
        torch.cuda.synchronize()
        c0 = rb.n_committed.clone()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            if name == "greedy":
                eng.round_launch(rb)
            else:
                sr.draft(smp)
                sr.verify(smp, st.rng)
        e1.record()
        torch.cuda.synchronize()
        eng.check_status(rb)
        ms = e0.elapsed_time(e1) / steps
        toks = int((rb.n_committed - c0).sum())
        out[name] = {"ms_per_round": round(ms, 4), "tokens_per_s": round(toks / (ms * steps / 1e3), 1),
                     "tokens_per_forward": round(toks / (2 * steps * bs), 4)}
    restore()
    out["params"] = "temperature 0.8, top_p 0.95, top_k 50, repetition 1.1, frequency 0.1 (joint filter), eager launches"
    return out


def e2e_worker(eng, rb, cfg, K, steps, dev, warmup):
    """Rounds through SelfSpecDiffusionWorker.forward_batch_generation: per round the scheduler's request slots
    are copied host->device from pinned memory, and the packed commit rows + status are read back (plus the host
    finish rules)."""
    from gravityocr_b200.compat.sglang_worker import ReqToPagePool, SelfSpecDiffusionWorker
    from gravityocr_b200.compat.types import ForwardMode, Req, SamplingParams, ScheduleBatch
    import types as _t
    bs = rb.bs
    pool = ReqToPagePool.__new__(ReqToPagePool)
    pool.engine, pool.size, pool.pages_per_req = eng, bs, rb.page_table.shape[1]
    pool.table, pool.owned = rb.page_table.clone(), {}
    target = _t.SimpleNamespace(engine=eng, req_to_page=pool)
    args = _t.SimpleNamespace(speculative_num_draft_tokens=K, page_size=16, model_path="", ss_draft_ahead=True)
    os.environ["SELFSPEC_MASK_ID"] = str(cfg.mask_id)
    wk = SelfSpecDiffusionWorker(args, 0, 0, None, 0, 0, 0, 0, target)
    wk._seeds().copy_(rb.seeds)
    reqs = []
    for b in range(bs):
        r = Req(b, torch.zeros((0, cfg.hidden)), [], SamplingParams(max_new_tokens=1 << 30), cfg.vocab)
        r._spec_seed_ready = True
        reqs.append(r)
    rpi_host = torch.arange(bs, dtype=torch.int64).pin_memory()
    rpi_dev = torch.empty((bs,), dtype=torch.int64, device=dev)
    batch = ScheduleBatch(reqs, rpi_dev, rb.seq_lens.clone(), ForwardMode.DECODE, rb.seq_lens.cpu())
    for _ in range(warmup):  # warm-up (the first call captures the worker's graph)
        rpi_dev.copy_(rpi_host, non_blocking=True)
        wk.forward_batch_generation(batch)
    torch.cuda.synchronize()
    wrb = wk._rb[bs]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    toks = 0
    e0.record()
    for _ in range(steps):
        rpi_dev.copy_(rpi_host, non_blocking=True)
        res = wk.forward_batch_generation(batch)
        toks += sum(len(t) for t in res.next_token_ids_cpu)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    # the state the rounds leave: K/V lengths, seed pool, committed tokens since the pre-warm-up state
    final = (wrb.seq_lens.cpu().tolist(), wrb.seeds.cpu().tolist(), wrb.n_committed.cpu().tolist())
    return {"value": None, "unit": "tokens/s", "h2d_bytes_per_step": bs * 8,
            "d2h_bytes_per_step": int(rb.readback.numel() * 4), "steps": steps,
            "api": "SelfSpecDiffusionWorker.forward_batch_generation (draft-ahead on)",
            "draft_ahead": dict(wk.ahead_stats), "tokens": toks, "ms": ms, "final": final}


def bs1_crop(eng, cfg, w, K, dev, hbm_peak):
    """Config 2 shape at batch 1 (prefix 256 + 32, 1024 generated tokens): natural mode and forced-accept replay
    (drafts overwritten from the natural stream so accept lengths are U{0..B}, seed 2)."""
    from gravityocr_b200.metrics import forward_bytes
    n_tok = 1024
    P = 256 + 32
    cap = P + 2 * n_tok + 4 * K + 64
    ppr = (cap + 15) // 16
    eng.reserve(K)
    rb = eng.new_round_buffers(1, K, ppr, max_len=cap, avg_len=P + n_tok // 2)
    pages = eng.pool.alloc(ppr)
    rb.page_table[0] = torch.tensor(pages, dtype=torch.int32, device=dev)
    x, ids = request_rows(cfg, w, 2, 0, 256)
    eng.prefill(rb, [x], [ids])
    snap = (rb.seq_lens.clone(), rb.seeds.clone(), rb.n_committed.clone(), rb.rounds.clone())

    def restore():
        rb.seq_lens.copy_(snap[0]); rb.seeds.copy_(snap[1]); rb.n_committed.copy_(snap[2]); rb.rounds.copy_(snap[3])

    eng.round_launch(rb)
    torch.cuda.synchronize()
    restore()
    gd, gv = eng.capture_split(rb)
    out = {}
    # natural mode: rounds until 1024 tokens are committed (device counters; one sync at the end)
    rounds = 0
    hist = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    d_ms = v_ms = 0.0
    while True:
        ta, tb, tc = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        ta.record(); gd.replay(); tb.record(); gv.replay(); tc.record()
        hist.append((ta, tb, tc))
        rounds += 1
        if rounds % 32 == 0 and int(rb.n_committed[0]) >= n_tok:
            break
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    d_ms = sum(a.elapsed_time(b) for a, b, c in hist) / rounds
    v_ms = sum(b.elapsed_time(c) for a, b, c in hist) / rounds
    n = int(rb.n_committed[0]) - 1
    S_mid = P + n // 2
    out["natural"] = {"tokens_per_s": round(n / (ms / 1000.0), 1), "tokens": n, "rounds": rounds,
                      "tokens_per_forward": round(n / (2 * rounds), 4), "draft_ms": round(d_ms, 4),
                      "verify_ms": round(v_ms, 4),
                      "hbm_frac_draft": round(forward_bytes(cfg, [S_mid], K, False) / (d_ms / 1e3) / (hbm_peak * 1e9), 4),
                      "hbm_frac_verify": round(forward_bytes(cfg, [S_mid], K, True) / (v_ms / 1e3) / (hbm_peak * 1e9), 4)}
    # the natural stream g, read from the committed rows of a replay with per-round readback
    restore()
    g = [int(rb.seeds[0])]
    while len(g) < n_tok + K + 2:
        gd.replay(); gv.replay()
        row = rb.packed[0].tolist()
        g += [row[0]] + row[2: 3 + row[1]]
    # forced-accept replay
    restore()
    gen = torch.Generator().manual_seed(2)
    plan = torch.randint(0, K, (1, 2 * n_tok), generator=gen, dtype=torch.int32)
    rb.override_g = torch.tensor([g + [0] * (2 * K)], dtype=torch.int32, device=dev)
    rb.override_plan = plan.to(dev)
    fd, fv = eng.capture_split(rb, override=True)
    restore()
    rounds = 0
    e0.record()
    while True:
        fd.replay(); fv.replay()
        rounds += 1
        if rounds % 16 == 0 and int(rb.n_committed[0]) >= n_tok:
            break
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    n = int(rb.n_committed[0]) - 1
    # untimed check of the same replay: every round accepts exactly its planned A_r and the stream is g
    restore()
    f_out, accs = [int(rb.seeds[0])], []
    while len(f_out) < n_tok:
        fd.replay(); fv.replay()
        row = rb.packed[0].tolist()
        accs.append(row[1])
        f_out += [row[0]] + row[2: 3 + row[1]]
    same = f_out == g[: len(f_out)] and accs == plan[0, : len(accs)].tolist()
    out["forced_accept"] = {"tokens_per_s": round(n / (ms / 1000.0), 1), "tokens": n, "rounds": rounds,
                            "tokens_per_forward": round(n / (2 * rounds), 4),
                            "plan": "A_r ~ U{0..16}, seed 2", "stream_equals_natural_and_accepts_plan": same}
    eng.pool.release(pages)
    out["workload"] = "config2-bs1-crop (prefix 256 + 32, 1024 tokens), weights of the config-3 replica"
    return out


def config4_sweep(a):
    """Config 4 (full-page long output): prefix 4096 image + 64 prompt tokens, B in {4, 8, 16, 32}, batch 1 and
    128 on one GPU; steady-state rounds after prefill (each B starts from the same post-prefill state).  Prints one
    JSON line with tokens/forward and % of the measured HBM roofline per draft and verify forward for each (B, batch).
    Bounded sample: `--steps` rounds per point instead of the full 4096 generated tokens."""
    from gravityocr_b200 import dp
    from gravityocr_b200.config import ModelConfig
    from gravityocr_b200.engine import Engine
    from gravityocr_b200.metrics import forward_bytes
    from gravityocr_b200.weights import random_weights
    rank, world, local = dp.dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    hbm_peak, _, _, peak_src = peaks()
    cfg = ModelConfig()
    w = random_weights(cfg, 4, torch.bfloat16)
    P = 4096 + 64
    steps = max(4, min(a.steps, 40))
    out = {"metric": METRIC, "config": {"workload": "config4-fullpage-sweep", "prefix": P, "steps_per_point": steps,
                                        "seed": 4, "peak_gbs": hbm_peak, "peak": peak_src}, "points": []}
    for bs in (1, 128):
        cap = P + (a.warmup + steps + 4) * 34 + 2 * 33 + 64
        ppr = (cap + 15) // 16
        eng = Engine(cfg, w, max_rows=max(bs * 33, bs * 64), n_pages=bs * ppr + 8, device=dev)
        rbs = {}
        pages = [eng.pool.alloc(ppr) for _ in range(bs)]
        xs, ids = zip(*[request_rows(cfg, w, 4, i, 4096, 64) for i in range(bs)])
        base = None
        for B in (4, 8, 16, 32):
            K = B + 1
            eng.reserve(bs * K)
            rb = eng.new_round_buffers(bs, K, ppr, max_len=cap, avg_len=P + 200)
            for b in range(bs):
                rb.page_table[b] = torch.tensor(pages[b], dtype=torch.int32, device=dev)
            if base is None:
                eng.prefill(rb, list(xs), list(ids))
                base = (rb.seq_lens.clone(), rb.seeds.clone())
            rb.seq_lens.copy_(base[0]); rb.seeds.copy_(base[1]); rb.n_committed.fill_(1)
            eng.refresh_order(rb)
            eng.round_launch(rb)
            torch.cuda.synchronize()
            rb.seq_lens.copy_(base[0]); rb.seeds.copy_(base[1]); rb.n_committed.fill_(1)
            gd, gv = eng.capture_split(rb)
            for _ in range(a.warmup):
                gd.replay(); gv.replay()
            torch.cuda.synchronize()
            c0 = rb.n_committed.clone()
            s0 = rb.seq_lens.cpu().tolist()
            total, dms, vms = time_graphs(gd, gv, steps)
            eng.check_status(rb)
            toks = int((rb.n_committed - c0).sum())
            s1 = rb.seq_lens.cpu().tolist()
            mid = [(x + y) / 2 for x, y in zip(s0, s1)]
            out["points"].append({
                "B": B, "batch": bs, "tokens_per_s": round(toks / (total / 1000.0), 1),
                "tokens_per_forward": round(toks / (2 * steps * bs), 4),
                "draft_ms": round(dms / steps, 4), "verify_ms": round(vms / steps, 4),
                "hbm_frac_draft": round(forward_bytes(cfg, mid, K, False) / (dms / steps / 1e3) / (hbm_peak * 1e9), 4),
                "hbm_frac_verify": round(forward_bytes(cfg, mid, K, True) / (vms / steps / 1e3) / (hbm_peak * 1e9), 4)})
            del gd, gv
        del eng
        torch.cuda.empty_cache()
    print(json.dumps(out), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------------------------------
# Single-kernel cases for ncu captures: `python bench.py case attention|linear|norm|sample|timeline ...`.  Each is a small,
# self-contained workload (a few GB on the device at most, inputs larger than L2): one untimed warm-up launch, then
# `--reps` launches; prints the mean CUDA-event time and the algorithmic bytes / FLOPs of one launch.  Example:
#
#     python bench.py case attention --bs 64 --mixed --reps 2
#     ncu --set full --clock-control none -k regex:attention_tc -s 1 -c 1 -o prof \
#         python bench.py case attention --bs 64 --mixed --reps 2
# ---------------------------------------------------------------------------------------------------------------------

def _case_time(fn, reps, graph):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
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
    else:
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def case_attention(a):
    """One attention launch over a paged cache: --seq tokens per request, or the config-3 prefix mix (--mixed)."""
    from gravityocr_b200 import _lib as L
    from gravityocr_b200.config import ModelConfig
    from gravityocr_b200.engine import attention_split
    from gravityocr_b200.metrics import attention_bytes
    cfg = ModelConfig()
    bs, K = a.bs, a.bd + 1
    g = torch.Generator().manual_seed(1)
    nq, nkv, D, ps = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, 16
    if a.mixed:
        S = (torch.randint(256, 4097, (bs,), generator=torch.Generator().manual_seed(SEED)) + 32).tolist()
    else:
        S = [a.seq] * bs
    seq_max = max(S)
    ppr = (seq_max + K + 2 + ps - 1) // ps
    n_pages = bs * ppr
    kc = torch.randn((n_pages, nkv, ps, D), generator=g).to("cuda", torch.bfloat16)
    vc = torch.randn((n_pages, nkv, ps, D), generator=g).to("cuda", torch.bfloat16)
    pt = torch.randperm(n_pages, generator=g).to(torch.int32).view(bs, ppr).cuda()
    seq = torch.tensor(S, dtype=torch.int64, device="cuda")
    q = torch.randn((bs * K, nq, D), generator=g).to("cuda", torch.bfloat16)
    out = torch.empty_like(q)
    chunk, splits = attention_split(bs, K, seq_max, sum(S) // len(S), nkv, L.num_sms())
    if a.chunk:
        chunk, splits = a.chunk, int(math.ceil((seq_max + K + 1) / a.chunk))
    ws = torch.zeros((L.attention_workspace_bytes(bs, K, nq, nkv, splits),), dtype=torch.uint8, device="cuda")
    order = torch.argsort(seq, descending=True, stable=True).to(torch.int32) if a.mixed else None
    base_add = 0 if a.draft else 1
    fn = lambda: L.bd_attention(q, kc, vc, pt, seq, bs, K, a.draft, base_add, nq, nkv, ps, chunk, splits, out, ws,
                                order=order)
    L.set_attention_tc(0 if a.mma else (2 if a.tc_all else 1))
    ms = _case_time(fn, a.reps, a.graph)
    b = attention_bytes(cfg, S, K, base_add)
    tc = not a.mma and nq // nkv * K <= 128 and (a.tc_all or bs * nkv * splits > L.num_sms())
    return {"kernel": "attention_tc_kernel" if tc else "attention_kernel", "bs": bs,
            "seq": "mixed" if a.mixed else a.seq, "K": K, "chunk": chunk, "splits": splits, "ms": ms, "bytes": b,
            "GBps": b / ms / 1e6}


def case_linear(a):
    """One projection launch: an [n_out, k_in] bf16 weight against m token rows with the chosen epilogue."""
    from gravityocr_b200 import _lib as L
    from gravityocr_b200.config import ModelConfig
    from gravityocr_b200.engine import rope_inv_freq
    cfg = ModelConfig()
    n_out, k_in, m = a.n_out, a.k_in, a.m
    g = torch.Generator().manual_seed(2)
    w = (torch.randn((n_out, k_in), generator=g) * 0.02).to("cuda", torch.bfloat16)
    x = torch.randn((m, k_in), generator=g).to("cuda", torch.bfloat16)
    mode = {"f32": L.EPI_STORE_F32, "bf16": L.EPI_STORE_BF16, "partial": L.EPI_PARTIAL_F32, "swiglu": L.EPI_SWIGLU,
            "argmax": L.EPI_ARGMAX, "qkv": L.EPI_QKV_ROPE}[a.epi]
    sp = a.splits or L.linear_default_splits(n_out, k_in, m, mode)
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
    elif mode == L.EPI_STORE_BF16:
        out = torch.zeros((m, n_out), dtype=torch.bfloat16, device="cuda")
        e.out, e.ld_out = out.data_ptr(), n_out
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
    ms = _case_time(lambda: L.linear(w, x, m, e, ws, splits=sp), a.reps, a.graph)
    fl = 2 * n_out * k_in * m
    return {"kernel": "linear_kernel", "epi": a.epi, "n_out": n_out, "k_in": k_in, "m": m, "splits": sp, "ms": ms,
            "weight_GBps": n_out * k_in * 2 / ms / 1e6, "TFLOPs": fl / ms / 1e9}


def case_norm(a):
    """One residual + sandwich norm launch over --m rows of hidden 1,536 summing --parts split-K partials."""
    from gravityocr_b200 import _lib as L
    m, H, sp = a.m, 1536, a.parts
    g = torch.Generator().manual_seed(3)
    y = (torch.randn((sp, m, H), generator=g) * 0.3).cuda()
    h = (torch.randn((m, H), generator=g) * 0.1).cuda()
    wa = (torch.randn((H,), generator=g) * 0.02).to("cuda", torch.bfloat16)
    wb = (torch.randn((H,), generator=g) * 0.02).to("cuda", torch.bfloat16)
    h2 = torch.empty_like(h)
    xo = torch.empty((m, H), dtype=torch.bfloat16, device="cuda")
    ms = _case_time(lambda: L.residual_norm(m, h, y, wa, wb, 1e-5, h2, xo, y_parts=sp), a.reps, a.graph)
    b = m * H * (4 * sp + 4 + 4 + 2)
    return {"kernel": "residual_norm", "m": m, "parts": sp, "ms": ms, "bytes": b, "GBps": b / ms / 1e6}


_TL_KINDS = {1: "attention_kernel", 2: "attention_tc_kernel", 3: "argmax_reduce_kernel", 4: "residual_norm",
             5: "penalty_cumulate_kernel", 6: "embed_rows_kernel", 7: "accept_commit_kernel",
             8: "logits_process_kernel", 9: "sample_rows_kernel", 10: "linear f32 (lm_head logits)", 11: "linear bf16",
             12: "linear gate_up+SwiGLU", 13: "linear QKV+RoPE", 14: "linear lm_head+argmax", 15: "linear o/down partials"}


def _timeline_records(lib):
    """(kind, block, entry, dependency release or 0, exit) per CTA, from every unit's record array: the release record
    of a CTA is the latest one of its block inside its [entry, exit] (an earlier kernel's CTA with the same block index
    may release inside that window too, but before it)."""
    import ctypes

    class Rec(ctypes.Structure):
        _fields_ = [("kind", ctypes.c_uint32), ("block", ctypes.c_uint32), ("t0", ctypes.c_uint64),
                    ("t1", ctypes.c_uint64)]
    out = []
    for unit in ("linear", "attention", "attention_tc", "rowwise", "sampling"):
        buf = (Rec * (1 << 19))()
        n = ctypes.c_uint32(0)
        assert getattr(lib, "gr_timeline_read_" + unit)(buf, ctypes.byref(n)) == 0
        rs = [(r.kind, r.block, r.t0, r.t1) for r in buf[:min(n.value, 1 << 19)]]
        deps = {}
        for r in rs:
            if r[0] == 0:
                deps.setdefault(r[1], []).append(r[2])
        for r in rs:
            if r[0]:
                d = [t for t in deps.get(r[1], ()) if r[2] <= t <= r[3]]
                out.append((r[0], r[1], r[2], max(d) if d else 0, r[3]))
    return out


def _timeline_launches(recs):
    """Group CTA records into launches: in entry order, a launch is a run of one kind with distinct blocks (the next
    kernel's CTAs start only after every CTA of this one has started)."""
    out = []
    for r in sorted(recs, key=lambda r: r[2]):
        if not (out and out[-1]["kind"] == r[0] and r[1] not in out[-1]["blocks"]):
            out.append({"kind": r[0], "blocks": set(), "t0": r[2], "dep": None, "t1": 0})
        L = out[-1]
        L["blocks"].add(r[1])
        L["t1"] = max(L["t1"], r[4])
        if r[3]:
            L["dep"] = r[3] if L["dep"] is None else min(L["dep"], r[3])
    return out


def case_timeline(a):
    """Live per-kernel timeline of one self-spec round (draft + verify + commit graphs) from the timeline build
    (python -m gravityocr_b200.build --timeline): per kernel kind, its share of the round (the time from the previous
    launch's last CTA exit to this launch's last exit), its critical path after its dependency was released, and the
    release latency.  Batch 1: the config-2 crop (prefix 288); larger batches: the first --batch config-3 requests.
    --sampled: a sampled round instead (eager launches, as the worker runs non-plain batches)."""
    os.environ.setdefault("GRAVITY_B200_LIB", os.path.join(ROOT, "gravityocr_b200", "libgravity_b200_timeline.so"))
    import ctypes
    from gravityocr_b200 import _lib as L
    from gravityocr_b200.config import ModelConfig
    from gravityocr_b200.engine import Engine
    from gravityocr_b200.weights import random_weights
    lib = ctypes.CDLL(L.LIB_PATH)
    cfg = ModelConfig()
    dev = torch.device("cuda", 0)
    K, bs = a.bd + 1, a.batch
    w = random_weights(cfg, SEED, torch.bfloat16)
    if bs == 1:
        P = 288
        cap = P + 2 * 1024 + 4 * K + 64
        ppr = (cap + 15) // 16
        eng = Engine(cfg, w, max_rows=64, n_pages=ppr + 16, device=dev)
        eng.reserve(K)
        rb = eng.new_round_buffers(1, K, ppr, max_len=cap, avg_len=P + 512)
        rb.page_table[0] = torch.tensor(eng.pool.alloc(ppr), dtype=torch.int32, device=dev)
        x, ids = request_rows(cfg, w, 2, 0, 256)
        eng.prefill(rb, [x], [ids])
    else:
        n_img, _ = workload(cfg, bs, SEED)
        prefix = [n_img[i] + 32 for i in range(bs)]
        cap = max(prefix) + 40 * (K + 1) + 2 * K + 64
        ppr = (cap + 15) // 16
        eng = Engine(cfg, w, max_rows=max(bs * K, bs * 64), n_pages=bs * ppr + 8, device=dev)
        eng.reserve(bs * K)
        rb = eng.new_round_buffers(bs, K, ppr, max_len=cap, avg_len=int(sum(prefix) / bs))
        for b in range(bs):
            rb.page_table[b] = torch.tensor(eng.pool.alloc(ppr), dtype=torch.int32, device=dev)
        xs, ids = zip(*[request_rows(cfg, w, SEED, i, n_img[i]) for i in range(bs)])
        eng.prefill(rb, list(xs), list(ids), chunk=64)
    eng.round_launch(rb)
    torch.cuda.synchronize()
    gd, gv = eng.capture_split(rb)
    for _ in range(4):
        gd.replay()
        gv.replay()
    torch.cuda.synchronize()
    if a.sampled:
        from gravityocr_b200.sampling import RequestSampling, SampledRound, SamplerState
        st = SamplerState(cfg.vocab, rb.seeds.shape[0], dev, seed=SEED)
        rs = [RequestSampling(temperature=0.8, top_p=0.95, top_k=50, repetition_penalty=1.1,
                              frequency_penalty=0.1)] * bs
        smp = st.batch(rs, rb.rpi)
        sr = SampledRound(eng, rb)
        for _ in range(2):
            sr.draft(smp)
            sr.verify(smp, st.rng)
        torch.cuda.synchronize()
    for unit in ("linear", "attention", "attention_tc", "rowwise", "sampling"):
        assert getattr(lib, "gr_timeline_clear_" + unit)() == 0
    if a.sampled:  # eager launches, as the worker runs a non-plain batch
        sr.draft(smp)
        sr.verify(smp, st.rng)
    else:
        gd.replay()
        gv.replay()
    torch.cuda.synchronize()
    eng.check_status(rb)
    ls = _timeline_launches(_timeline_records(lib))
    agg = {}
    prev = ls[0]["t0"]
    for L_ in ls:
        name = _TL_KINDS.get(L_["kind"], str(L_["kind"]))
        dep = L_["dep"] or L_["t0"]
        g = agg.setdefault(name, {"launches": 0, "round_us": 0.0, "busy_us": 0.0, "release_us": 0.0})
        g["launches"] += 1
        g["round_us"] += (L_["t1"] - prev) / 1e3
        g["busy_us"] += (L_["t1"] - dep) / 1e3
        g["release_us"] += (dep - prev) / 1e3
        prev = L_["t1"]
    total = (ls[-1]["t1"] - ls[0]["t0"]) / 1e3
    kinds = {}
    for name, g in sorted(agg.items(), key=lambda kv: -kv[1]["round_us"]):
        n = g["launches"]
        kinds[name] = {"launches": n, "round_us": round(g["round_us"], 1), "share": round(g["round_us"] / total, 4),
                       "avg_us": round(g["round_us"] / n, 2), "avg_busy_us": round(g["busy_us"] / n, 2),
                       "avg_release_us": round(g["release_us"] / n, 2)}
    return {"case": "timeline", "batch": bs, "K": K, "sampled": bool(a.sampled), "launches": len(ls),
            "round_us": round(total, 1),
            "forward_us": round(total / 2, 1), "kinds": kinds,
            "note": "avg_us: launch share of the round (previous launch's last exit to this one's); avg_busy_us: "
                    "dependency release to last CTA exit (PDL lets a launch's CTAs start before that); "
                    "avg_release_us: previous launch's last exit to this launch's first griddepcontrol.wait return"}


def case_sample(a):
    """One sample_rows launch over bs x K verify rows of fp32 logits (vocabulary 59,392): temperature 0.8, top-k 50,
    top-p 0.95 under the joint filter (or --filter), accept bits against seeded draft tokens and the draws."""
    from gravityocr_b200 import _lib as L
    from gravityocr_b200.config import ModelConfig
    from gravityocr_b200.sampling import RequestSampling, SamplerState
    cfg = ModelConfig()
    bs, K, V = a.bs, a.bd + 1, cfg.vocab
    g = torch.Generator().manual_seed(5)
    logits = (torch.randn((bs * K, V), generator=g) * a.scale).cuda()
    cand = torch.randint(0, V, (bs * K,), generator=g).to("cuda", torch.int32)
    rpi = torch.arange(bs, dtype=torch.int64, device="cuda")
    flt = {"joint": L.FILTER_JOINT, "sequential": L.FILTER_SEQUENTIAL, "torch": L.FILTER_TORCH}[a.filter]
    st = SamplerState(V, bs, "cuda", seed=SEED, filter=flt)
    rs = [RequestSampling(temperature=0.8, top_k=a.top_k, top_p=a.top_p, min_p=a.min_p)] * bs
    smp = st.batch(rs, rpi)
    accept = torch.zeros((bs * K,), dtype=torch.int32, device="cuda")
    sample = torch.zeros((bs * K,), dtype=torch.int32, device="cuda")
    p_next = torch.zeros((bs * K,), dtype=torch.float32, device="cuda")
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    work = logits.clone()

    def fn():   # the kernel scales its rows in place, so each launch starts from a fresh copy
        work.copy_(logits)
        L.sample_rows(work, bs, K, cand, smp, L.COIN_FIRST, accept, sample, p_next, status=status)
    ms = _case_time(fn, a.reps, a.graph)
    assert int(status.item()) == 0
    return {"kernel": "sample_rows_kernel", "rows": bs * K, "vocab": V, "filter": a.filter, "top_k": a.top_k,
            "top_p": a.top_p, "ms_with_copy": ms, "logit_bytes": bs * K * V * 4}


def case_process(a):
    """One logits_process launch over bs x K verify rows of fp32 logits (vocabulary 59,392): repetition 1.1 and
    frequency 0.1 from seeded penalizer state, the in-block draft ids counted per row."""
    from gravityocr_b200 import _lib as L
    from gravityocr_b200.config import ModelConfig
    from gravityocr_b200.sampling import RequestSampling, SamplerState
    cfg = ModelConfig()
    bs, K, V = a.bs, a.bd + 1, cfg.vocab
    g = torch.Generator().manual_seed(6)
    logits = (torch.randn((bs * K, V), generator=g) * 3.0).cuda()
    cand = torch.randint(0, V, (bs * K,), generator=g).to("cuda", torch.int32)
    rpi = torch.arange(bs, dtype=torch.int64, device="cuda")
    st = SamplerState(V, bs, "cuda", seed=SEED)
    seen = torch.rand((bs, V), generator=g) < 0.01   # about 1% of the vocabulary already generated per request
    st.st_rep.copy_(torch.where(seen, 1.1, 1.0).cuda())
    st.st_freq.copy_(torch.where(seen, 0.1, 0.0).cuda())
    rs = [RequestSampling(temperature=0.8, top_k=50, top_p=0.95, repetition_penalty=a.repetition,
                          frequency_penalty=a.frequency)] * bs
    smp = st.batch(rs, rpi)
    work = logits.clone()

    def fn():   # the kernel rewrites its rows in place, so each launch starts from a fresh copy
        work.copy_(logits)
        L.logits_process(work, bs, K, cand, smp)
    ms = _case_time(fn, a.reps, a.graph)
    return {"kernel": "logits_process_kernel", "rows": bs * K, "vocab": V, "repetition": a.repetition,
            "frequency": a.frequency, "ms_with_copy": ms, "logit_bytes": bs * K * V * 4}


def case_main(argv):
    ap = argparse.ArgumentParser(prog="bench.py case")
    ap.add_argument("--graph", action="store_true", help="time launches captured in one CUDA graph")
    sub = ap.add_subparsers(dest="case", required=True)
    at = sub.add_parser("attention")
    at.add_argument("--bs", type=int, default=16)
    at.add_argument("--seq", type=int, default=2048)
    at.add_argument("--bd", type=int, default=K_BD)
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
    li.add_argument("--epi", default="swiglu", choices=["f32", "bf16", "partial", "swiglu", "argmax", "qkv"])
    li.add_argument("--splits", type=int, default=0)
    li.add_argument("--reps", type=int, default=3)
    nm = sub.add_parser("norm")
    nm.add_argument("--m", type=int, default=1088)
    nm.add_argument("--parts", type=int, default=2)
    nm.add_argument("--reps", type=int, default=3)
    tl = sub.add_parser("timeline")
    tl.add_argument("--batch", type=int, default=1)
    tl.add_argument("--bd", type=int, default=K_BD)
    tl.add_argument("--sampled", action="store_true",
                    help="a sampled round (temperature 0.8, top-k 50, top-p 0.95, penalties), eager launches")
    sa = sub.add_parser("sample")
    sa.add_argument("--bs", type=int, default=64)
    sa.add_argument("--bd", type=int, default=K_BD)
    sa.add_argument("--filter", default="joint", choices=["joint", "sequential", "torch"])
    sa.add_argument("--top-k", type=int, default=50)
    sa.add_argument("--top-p", type=float, default=0.95)
    sa.add_argument("--min-p", type=float, default=0.0)
    sa.add_argument("--scale", type=float, default=3.0, help="std of the synthetic logits")
    sa.add_argument("--reps", type=int, default=3)
    pr = sub.add_parser("process")
    pr.add_argument("--bs", type=int, default=64)
    pr.add_argument("--bd", type=int, default=K_BD)
    pr.add_argument("--repetition", type=float, default=1.1)
    pr.add_argument("--frequency", type=float, default=0.1)
    pr.add_argument("--reps", type=int, default=3)
    a = ap.parse_args(argv)
    fn = {"attention": case_attention, "linear": case_linear, "norm": case_norm, "sample": case_sample,
          "process": case_process, "timeline": case_timeline}[a.case]
    print(json.dumps(fn(a)), flush=True)
    return 0


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "case":
        sys.exit(case_main(sys.argv[2:]))
    sys.exit(main())
