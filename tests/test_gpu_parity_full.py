"""Full-depth (16-layer) round lockstep of the CUDA path against the fp32 oracle, at the shapes the benchmark runs.

* Config-3 subset: the benchmark's own weights (seed 3) and its first 8 requests (prefixes U[256, 4096] image tokens +
  32 prompt tokens, seed 3), batch 8, B = 16, the benchmark's attention plan (split KV with more CTAs than SMs: the
  tcgen05 kernel merging through global scratch) and longest-first launch order, 4 rounds.
* B sweep: B in {4, 8, 16, 32} (K = 5, 9, 17, 33) on the same model with its token-embedding table at std 0.25, whose
  greedy streams stay varied (at 0.02 they settle on one repeated token), so rejections and rollbacks occur; batch 4
  of config-3 prefixes, 4 rounds per B, every B starting from the same post-prefill state.

Every round, for every request, the oracle recomputes the draft and verify logits in fp32 from the same committed
tokens (its own fp32 K/V cache) and then follows the GPU's tokens (lockstep):
  * every GPU argmax equals the oracle's argmax, or is a listed near-tie (oracle top-2 gap < 1e-3);
  * every GPU top-1 logit is within 2e-2 of the oracle's, relative to the row's largest logit magnitude;
  * the commit is exact given the same argmaxes: packed row, seq_lens, seed pool, released positions.
The oracle runs its torch fp32 code on the GPU (TF32 off) so that 4k-token prefixes stay fast; it is the same
restatement the CPU tests pin to the reference."""
import pytest
import torch

from gravityocr_b200.config import ModelConfig
from gravityocr_b200.engine import Engine
from gravityocr_b200.weights import random_weights, request_inputs
from oracle.commit_ref import released_positions
from oracle.decoder_ref import OracleCache, OracleDecoder, SpecState, spec_commit, spec_draft, spec_verify

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIE = 1e-3
LOGIT_TOL = 2e-2
SEED = 3


def _requests(cfg, w_bf16, n, seed=SEED, n_prompt=32):
    """The benchmark's request list (bench.py workload + request_rows): layer-0 rows and ids of the first n."""
    g = torch.Generator().manual_seed(seed)
    n_img = torch.randint(256, 4097, (64,), generator=g).tolist()
    out = []
    for i in range(n):
        img, txt = request_inputs(cfg, seed, n_img[i], n_prompt, i, torch.bfloat16)
        x = torch.cat([img, w_bf16["embed_tokens"][txt].float()], 0)
        ids = torch.cat([torch.full((n_img[i],), -1, dtype=torch.int64), txt])
        out.append((x, ids))
    return out


class _Lockstep:
    def __init__(self):
        self.ties = []
        self.rows = 0

    def rows_check(self, name, gpu_idx, gpu_top, lg):
        o = torch.topk(lg.float(), 2, dim=-1)
        oi, gap = o.indices[:, 0].cpu(), (o.values[:, 0] - o.values[:, 1]).cpu()
        top = o.values[:, 0].cpu()
        self.rows += lg.shape[0]
        for r in range(lg.shape[0]):
            if int(gpu_idx[r]) != int(oi[r]):
                assert float(gap[r]) < TIE, \
                    f"{name} row {r}: gpu {int(gpu_idx[r])} oracle {int(oi[r])} gap {float(gap[r]):.2e}"
                self.ties.append((name, r, float(gap[r])))
        scale = lg.abs().max(dim=-1).values.cpu()
        err = (gpu_top - top).abs()
        assert bool((err <= LOGIT_TOL * scale).all()), f"{name}: top-1 logit off by {float((err / scale).max()):.3e}"


def _setup(cfg, w, reqs, K, rounds):
    bs = len(reqs)
    P = [x.shape[0] for x, _ in reqs]
    cap = max(P) + rounds * (33 + 1) + 2 * 33 + 64
    ppr = (cap + 15) // 16
    eng = Engine(cfg, w, max_rows=max(bs * 33, bs * 64), n_pages=bs * ppr + 8)
    eng.reserve(bs * 33)
    pages = [eng.pool.alloc(ppr) for _ in range(bs)]
    return eng, pages, ppr, cap, P


def _buffers(eng, pages, ppr, cap, P, K):
    rb = eng.new_round_buffers(len(pages), K, ppr, max_len=cap, avg_len=int(sum(P) / len(P)))
    for b, pg in enumerate(pages):
        rb.page_table[b] = torch.tensor(pg, dtype=torch.int32, device=DEV)
    return rb


def _oracle_states(oracle, reqs, cap):
    sts = []
    for x, _ in reqs:
        cache, lg = oracle.prefill(x.to(DEV), cap)
        s = int(lg.argmax())
        sts.append((SpecState(cache, x.shape[0], s, [s], x.shape[0]), lg))
    return sts


def _lockstep_rounds(eng, rb, oracle, states, first, K, rounds, ls):
    bs = rb.bs
    for b, (st, lg) in enumerate(states):
        if first[b] != st.seed:   # the prefill's first token: a near-tie at most, then follow the GPU
            t2 = torch.topk(lg, 2).values
            assert float(t2[0] - t2[1]) < TIE, f"request {b}: prefill token differs beyond a near-tie"
            ls.ties.append(("prefill", b, float(t2[0] - t2[1])))
            st.seed = first[b]
            st.out = [first[b]]
    accs = []
    for r in range(rounds):
        s_before = [st.seq_len for st, _ in states]
        assert rb.seq_lens.cpu().tolist() == s_before
        eng.round_launch(rb)
        torch.cuda.synchronize()
        eng.check_status(rb)
        am, v = rb.am.cpu().view(bs, K), rb.v.cpu().view(bs, K)
        top_d, top_v = rb.top_d.cpu().view(bs, K), rb.top_v.cpu().view(bs, K)
        pk = rb.packed.cpu()
        rel_all = []
        for b, (st, _) in enumerate(states):
            _, dlg = spec_draft(oracle, st, K)
            ls.rows_check(f"K{K} r{r} b{b} draft", am[b], top_d[b], dlg)
            _, vlg = spec_verify(oracle, st, am[b].long().to(DEV))
            ls.rows_check(f"K{K} r{r} b{b} verify", v[b], top_v[b], vlg)
            res = spec_commit(st, am[b].tolist(), v[b].tolist())
            acc = res["acc"]
            accs.append(acc)
            row = pk[b].tolist()
            assert row[0] == int(am[b, 0]) and row[1] == acc
            assert row[2: 3 + acc] == v[b, : acc + 1].tolist() and not any(row[3 + acc:])
            rel_all += released_positions(s_before[b], acc, K)
        assert rb.seq_lens.cpu().tolist() == [st.seq_len for st, _ in states]
        assert rb.seeds.cpu()[rb.rpi.cpu()].tolist() == [st.seed for st, _ in states]
        n_rel = int(rb.n_released[0])
        assert rb.released[:n_rel].cpu().tolist() == rel_all
    return accs


@pytest.fixture(scope="module")
def fp32_exact():
    prev = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev


def test_config3_subset_lockstep_16_layers(fp32_exact):
    cfg = ModelConfig()
    K, rounds, bs = 17, 4, 8
    w = random_weights(cfg, SEED, torch.bfloat16)
    reqs = _requests(cfg, w, bs)
    eng, pages, ppr, cap, P = _setup(cfg, w, reqs, K, rounds)
    rb = _buffers(eng, pages, ppr, cap, P, K)
    assert rb.attn_splits > 1 and bs * cfg.n_kv_heads * rb.attn_splits > eng.sms  # split KV, global merge
    first = eng.prefill(rb, [x for x, _ in reqs], [i for _, i in reqs])
    assert rb.order.cpu().tolist() == sorted(range(bs), key=lambda b: (-P[b], b))   # longest first
    oracle = OracleDecoder(cfg, {k: t.float() for k, t in w.items()}, device=DEV)
    states = _oracle_states(oracle, reqs, cap)
    ls = _Lockstep()
    _lockstep_rounds(eng, rb, oracle, states, first, K, rounds, ls)
    # every mismatch was asserted to be an fp32 near-tie; with the baseline's 0.02 embedding table some requests settle
    # on rows whose two best tokens are tied within 1e-4, so the listing can be long
    print(f"config-3 subset: {ls.rows} rows checked, {len(ls.ties)} near-ties listed: {ls.ties}")


def test_block_size_sweep_lockstep_16_layers(fp32_exact):
    cfg = ModelConfig()
    rounds, bs = 4, 4
    w = random_weights(cfg, SEED, torch.bfloat16, embed_std=0.25)
    reqs = _requests(cfg, w, bs)
    eng, pages, ppr, cap, P = _setup(cfg, w, reqs, 33, rounds)
    oracle = OracleDecoder(cfg, {k: t.float() for k, t in w.items()}, device=DEV)
    base, first, snap = None, None, None
    ls = _Lockstep()
    accs_all = {}
    for B in (4, 8, 16, 32):
        K = B + 1
        rb = _buffers(eng, pages, ppr, cap, P, K)
        if base is None:
            first = eng.prefill(rb, [x for x, _ in reqs], [i for _, i in reqs])
            base = (rb.seq_lens.clone(), rb.seeds.clone())
            states = _oracle_states(oracle, reqs, cap)
            snap = [(st.cache.k.clone(), st.cache.v.clone(), lg) for st, lg in states]
        else:
            rb.seq_lens.copy_(base[0])
            rb.seeds.copy_(base[1])
            rb.n_committed.fill_(1)
            eng.refresh_order(rb)
            states = []
            for (k, v, lg), (x, _) in zip(snap, reqs):
                s = int(lg.argmax())
                st = SpecState(OracleCache(k.clone(), v.clone()), x.shape[0], s, [s], x.shape[0])
                states.append((st, lg))
        accs_all[B] = _lockstep_rounds(eng, rb, oracle, states, first, K, rounds, ls)
        del rb
    print(f"B sweep: {ls.rows} rows checked, accept lengths {accs_all}, {len(ls.ties)} near-ties listed: {ls.ties}")
