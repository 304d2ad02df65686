"""ctypes binding of ``libgravity_b200.so`` (C ABI in ``include/gravity_b200.h``).

The wrappers take torch tensors, check dtype / device / contiguity, pass raw device pointers and the current CUDA
stream, and raise ``RuntimeError`` on any non-zero status.  There is no fallback: if the library is missing or
fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("GRAVITY_B200_LIB", os.path.join(_HERE, "libgravity_b200.so"))

GR_OK = 0
EPI_STORE_F32, EPI_STORE_BF16, EPI_SWIGLU, EPI_QKV_ROPE, EPI_ARGMAX, EPI_PARTIAL_F32 = range(6)
ROWS_DRAFT, ROWS_VERIFY, ROWS_EXPLICIT = range(3)

# every symbol include/gravity_b200.h declares
EXPORTS = ("gr_version", "gr_status_string", "gr_set_pdl", "gr_set_attention_tc", "gr_num_sms", "gr_linear_workspace_bytes",
           "gr_attention_workspace_bytes", "gr_linear_default_splits", "gr_linear_plan", "gr_linear", "gr_embed_rows",
           "gr_residual_norm", "gr_bd_attention", "gr_accept_commit", "gr_draft_override", "gr_pack_gate_up",
           "gr_bd_attention_noalloc", "gr_bd_attention_ordered", "gr_gather_rows", "gr_logits_process",
           "gr_sample_rows", "gr_commit_sampled", "gr_penalty_cumulate")
FILTER_JOINT, FILTER_SEQUENTIAL, FILTER_TORCH = range(3)
PEN_REPETITION, PEN_FREQUENCY, PEN_PRESENCE, PEN_MIN_NEW_TOKENS = range(4)
COIN_ACCEPT, COIN_FINAL, COIN_FIRST, COIN_PREFILL = range(4)
GR_ERR_NO_TOKEN = 9


class Epilogue(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int),
        ("out", ctypes.c_void_p),
        ("ld_out", ctypes.c_int),
        ("q_out", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("row_pos", ctypes.c_void_p),
        ("row_slot", ctypes.c_void_p),
        ("inv_freq", ctypes.c_void_p),
        ("rotary_dim", ctypes.c_int),
        ("n_q_heads", ctypes.c_int),
        ("n_kv_heads", ctypes.c_int),
        ("page_size", ctypes.c_int),
        ("out_idx", ctypes.c_void_p),
        ("out_top1", ctypes.c_void_p),
        ("out_gap", ctypes.c_void_p),
        ("row_pos3", ctypes.c_void_p),
        ("mrope_section", ctypes.c_int * 3),
    ]


class Sampling(ctypes.Structure):
    """gr_sampling: per-request parameter arrays, penalizer state by pool slot, grammar mask, bias and the coins' rng."""
    _fields_ = [
        ("vocab", ctypes.c_int),
        ("filter", ctypes.c_int),
        ("temperature", ctypes.c_void_p),
        ("top_k", ctypes.c_void_p),
        ("top_p", ctypes.c_void_p),
        ("min_p", ctypes.c_void_p),
        ("n_order", ctypes.c_int),
        ("order", ctypes.c_int * 4),
        ("repetition", ctypes.c_void_p),
        ("frequency", ctypes.c_void_p),
        ("presence", ctypes.c_void_p),
        ("min_new_tokens", ctypes.c_void_p),
        ("stop_ids", ctypes.c_void_p),
        ("n_stop", ctypes.c_int),
        ("st_rep", ctypes.c_void_p),
        ("st_freq", ctypes.c_void_p),
        ("st_pres", ctypes.c_void_p),
        ("st_len", ctypes.c_void_p),
        ("req_pool_idx", ctypes.c_void_p),
        ("allowed", ctypes.c_void_p),
        ("logit_bias", ctypes.c_void_p),
        ("rng", ctypes.c_void_p),
    ]


_lib = None
_lock = threading.Lock()

_P, _I, _Z, _F, _L = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_float, ctypes.c_int64
_SIGS = {
    "gr_version": (_I, []),
    "gr_status_string": (ctypes.c_char_p, [_I]),
    "gr_set_pdl": (None, [_I]),
    "gr_set_attention_tc": (None, [_I]),
    "gr_num_sms": (_I, []),
    "gr_linear_workspace_bytes": (_Z, [_I, _I, _I]),
    "gr_attention_workspace_bytes": (_Z, [_I, _I, _I, _I, _I]),
    "gr_linear_default_splits": (_I, [_I, _I, _I, _I]),
    "gr_linear_plan": (_I, [_I, _I, _I, _I, _I, _P]),
    "gr_linear": (_I, [_P, _I, _I, _P, _I, ctypes.POINTER(Epilogue), _I, _P, _Z, _P, _Z, _P, _P]),
    "gr_embed_rows": (_I, [_I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _I, _I, _P, _F, _I, _P, _P, _P,
                           _P, _P, _P, _P, _P]),
    "gr_residual_norm": (_I, [_I, _I, _P, _P, _I, _P, _P, _F, _P, _P, _P]),
    "gr_bd_attention": (_I, [_P, _P, _P, _L, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _Z, _P, _P]),
    "gr_accept_commit": (_I, [_I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "gr_draft_override": (_I, [_I, _I, _P, _P, _I, _P, _P, _I, _P, _I, _I, _P]),
    "gr_pack_gate_up": (_I, [_P, _P, _I, _I, _P]),
    "gr_bd_attention_noalloc": (_I, [_P, _P, _P, _L, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "gr_gather_rows": (_I, [_P, _I, _I, _I, _P, _P]),
    "gr_logits_process": (_I, [_P, _I, _I, _P, ctypes.POINTER(Sampling), _P]),
    "gr_sample_rows": (_I, [_P, _I, _I, _P, ctypes.POINTER(Sampling), _I, _P, _P, _P, _P, _I, _P, _P]),
    "gr_commit_sampled": (_I, [_I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "gr_penalty_cumulate": (_I, [_I, _P, _I, _P, _I, ctypes.POINTER(Sampling), _P]),
    "gr_bd_attention_ordered": (_I, [_P, _P, _P, _L, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _Z, _P,
                                     _P]),
}
GR_ERR_SCRATCH_LIMIT = 8
NOALLOC_SCRATCH_BYTES = 8 << 20


def load(path: Optional[str] = None):
    """Load the library (once).  Raises if it is missing: there is no CPU or library fallback."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(f"libgravity_b200.so not found at {p}: build it with `python -m gravityocr_b200.build`")
        lib = ctypes.CDLL(p)
        for name, (res, args) in _SIGS.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
        return lib


def _check(rc: int, what: str) -> None:
    if rc != GR_OK:
        raise RuntimeError(f"{what} failed: {load().gr_status_string(rc).decode()} (code {rc})")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


# ---------------------------------------------------------------------- wrappers
def set_pdl(enable: bool) -> None:
    load().gr_set_pdl(1 if enable else 0)


def set_attention_tc(mode) -> None:
    """Attention kernel: 0 / False mma.sync everywhere; 1 / True tcgen05 on grids of more than one CTA per SM (the
    default); 2 tcgen05 on every grid."""
    load().gr_set_attention_tc(int(mode))


def num_sms() -> int:
    return int(load().gr_num_sms())


def linear_workspace_bytes(n_out: int, m: int, splits: int) -> int:
    return int(load().gr_linear_workspace_bytes(n_out, m, splits))


def linear_default_splits(n_out: int, k_in: int, m: int, mode: int = EPI_STORE_F32) -> int:
    """Split-K count gr_linear plans for this shape and epilogue mode."""
    return int(load().gr_linear_default_splits(n_out, k_in, m, mode))


def linear_plan(n_out: int, k_in: int, m: int, mode: int = EPI_STORE_F32, splits: int = 0) -> dict:
    """The plan gr_linear runs for this call: split count, token-tile height and count, unit order, grid."""
    out = (ctypes.c_int32 * 5)()
    _check(load().gr_linear_plan(n_out, k_in, m, mode, splits, out), "gr_linear_plan")
    return {"splits": out[0], "nt": out[1], "m_tiles": out[2], "tail_last": bool(out[3]), "grid": out[4]}


def attention_workspace_bytes(bs: int, K: int, n_q_heads: int, n_kv_heads: int, max_splits: int) -> int:
    return int(load().gr_attention_workspace_bytes(bs, K, n_q_heads, n_kv_heads, max_splits))


def linear(w: torch.Tensor, x: torch.Tensor, m: int, epi: Epilogue, workspace: torch.Tensor, splits: int = 0,
           prefetch: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None, stream=None) -> None:
    _need(w, torch.bfloat16, "w")
    _need(x, torch.bfloat16, "x")
    n_out, k_in = w.shape
    if x.shape[-1] != k_in or x.numel() < m * k_in:
        raise RuntimeError(f"x shape {tuple(x.shape)} does not match w {tuple(w.shape)} with m={m}")
    rc = load().gr_linear(w.data_ptr(), n_out, k_in, x.data_ptr(), m, ctypes.byref(epi), splits,
                          workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                          _ptr(prefetch), 0 if prefetch is None else prefetch.numel() * prefetch.element_size(),
                          _ptr(status), _stream(stream))
    _check(rc, "gr_linear")


def embed_rows(mode: int, bs: int, K: int, *, seeds=None, rpi=None, ids32=None, ids64=None, row_embeds=None,
               seq_lens, page_table, page_size: int, embed, vocab: int, mask_id: int, norm_w, eps: float,
               h_out, x_out, row_pos, row_slot, row_ids=None, rope_delta=None, status=None, stream=None) -> None:
    rc = load().gr_embed_rows(mode, bs, K, _ptr(seeds), _ptr(rpi), _ptr(ids32), _ptr(ids64), _ptr(row_embeds),
                              seq_lens.data_ptr(), page_table.data_ptr(), page_table.shape[1], page_size,
                              page_table.shape[1], embed.data_ptr(), vocab, mask_id, norm_w.data_ptr(), eps,
                              embed.shape[1], h_out.data_ptr(), x_out.data_ptr(), row_pos.data_ptr(),
                              row_slot.data_ptr(), _ptr(row_ids), _ptr(rope_delta), _ptr(status), _stream(stream))
    _check(rc, "gr_embed_rows")


def residual_norm(m: int, h_in, y, w_a, w_b, eps: float, h_out, x_out, y_parts: int = 1, stream=None) -> None:
    rc = load().gr_residual_norm(m, h_in.shape[-1], h_in.data_ptr(), y.data_ptr(), y_parts, w_a.data_ptr(),
                                 w_b.data_ptr(), eps, h_out.data_ptr(), x_out.data_ptr(), _stream(stream))
    _check(rc, "gr_residual_norm")


def bd_attention(q, k_cache, v_cache, page_table, seq_lens, bs: int, K: int, draft, base_add: int,
                 n_q_heads: int, n_kv_heads: int, page_size: int, chunk: int, max_splits: int, out, workspace,
                 status=None, stream=None, order=None) -> None:
    n_pages = k_cache.shape[0]
    rc = load().gr_bd_attention_ordered(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), n_pages,
                                page_table.data_ptr(), page_table.shape[1], seq_lens.data_ptr(), _ptr(order),
                                bs, K, int(draft), base_add,
                                n_q_heads, n_kv_heads, page_size, chunk, max_splits, out.data_ptr(),
                                _ptr(workspace), 0 if workspace is None else workspace.numel() * workspace.element_size(),
                                _ptr(status), _stream(stream))
    _check(rc, "gr_bd_attention")


def accept_commit(bs: int, K: int, am, v, seeds, rpi, seq_lens, packed, released, out_next, *, x0_committed=False,
                  loc=None, n_released=None, n_committed=None, rounds=None, accept_len=None, stream=None) -> None:
    rc = load().gr_accept_commit(bs, K, am.data_ptr(), v.data_ptr(), seeds.data_ptr(), rpi.data_ptr(),
                                 seq_lens.data_ptr(), 1 if x0_committed else 0, _ptr(loc), packed.data_ptr(),
                                 released.data_ptr(), _ptr(n_released), out_next.data_ptr(), _ptr(n_committed),
                                 _ptr(rounds), _ptr(accept_len), _stream(stream))
    _check(rc, "gr_accept_commit")


def draft_override(bs: int, K: int, am, g, n_committed, plan, rounds, vocab: int, mask_id: int, stream=None) -> None:
    rc = load().gr_draft_override(bs, K, am.data_ptr(), g.data_ptr(), g.shape[1], n_committed.data_ptr(),
                                  plan.data_ptr(), plan.shape[1], rounds.data_ptr(), vocab, mask_id, _stream(stream))
    _check(rc, "gr_draft_override")


def pack_gate_up(src: torch.Tensor, dst: torch.Tensor, intermediate: int, stream=None) -> None:
    _need(src, torch.bfloat16, "src")
    _need(dst, torch.bfloat16, "dst")
    rc = load().gr_pack_gate_up(src.data_ptr(), dst.data_ptr(), intermediate, src.shape[1], _stream(stream))
    _check(rc, "gr_pack_gate_up")


def bd_attention_noalloc(q, k_cache, v_cache, page_table, seq_lens, bs: int, K: int, draft, base_add: int,
                         n_q_heads: int, n_kv_heads: int, page_size: int, chunk: int, max_splits: int, out,
                         status=None, stream=None) -> None:
    """``bd_attention`` for callers that cannot allocate device memory: the split scratch is the library's own
    fixed 8 MiB device array (see ``gr_bd_attention_noalloc`` in include/gravity_b200.h for the limits)."""
    rc = load().gr_bd_attention_noalloc(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
                                        page_table.data_ptr(), page_table.shape[1], seq_lens.data_ptr(), bs, K,
                                        int(draft), base_add, n_q_heads, n_kv_heads, page_size, chunk,
                                        max_splits, out.data_ptr(), _ptr(status), _stream(stream))
    _check(rc, "gr_bd_attention_noalloc")


# ---------------------------------------------------------------------- non-greedy rounds
def gather_rows(src: torch.Tensor, n: int, stride_rows: int, dst: torch.Tensor, stream=None) -> None:
    row_bytes = src.shape[-1] * src.element_size()
    _check(load().gr_gather_rows(src.data_ptr(), row_bytes, n, stride_rows, dst.data_ptr(), _stream(stream)),
           "gr_gather_rows")


def logits_process(logits: torch.Tensor, bs: int, K: int, cand, smp: Sampling, stream=None) -> None:
    _need(logits, torch.float32, "logits")
    _check(load().gr_logits_process(logits.data_ptr(), bs, K, _ptr(cand), ctypes.byref(smp), _stream(stream)),
           "gr_logits_process")


def sample_rows(logits: torch.Tensor, bs: int, K: int, cand, smp: Sampling, first_kind: int, accept, sample,
                p_next=None, first_out=None, first_stride: int = 1, status=None, stream=None) -> None:
    _need(logits, torch.float32, "logits")
    _check(load().gr_sample_rows(logits.data_ptr(), bs, K, _ptr(cand), ctypes.byref(smp), first_kind, _ptr(accept),
                                 sample.data_ptr(), _ptr(p_next), _ptr(first_out), first_stride, _ptr(status),
                                 _stream(stream)), "gr_sample_rows")


def commit_sampled(bs: int, K: int, am, accept, sample, seeds, rpi, seq_lens, predict, packed, released, out_next, *,
                   n_released=None, n_committed=None, rounds=None, accept_len=None, rng=None, stream=None) -> None:
    _check(load().gr_commit_sampled(bs, K, am.data_ptr(), accept.data_ptr(), sample.data_ptr(), seeds.data_ptr(),
                                    rpi.data_ptr(), seq_lens.data_ptr(), predict.data_ptr(), packed.data_ptr(),
                                    released.data_ptr(), _ptr(n_released), out_next.data_ptr(), _ptr(n_committed),
                                    _ptr(rounds), _ptr(accept_len), _ptr(rng), _stream(stream)), "gr_commit_sampled")


def penalty_cumulate(bs: int, tokens, stride: int, counts, add: int, smp: Sampling, stream=None) -> None:
    _check(load().gr_penalty_cumulate(bs, tokens.data_ptr(), stride, _ptr(counts), add, ctypes.byref(smp),
                                      _stream(stream)), "gr_penalty_cumulate")
