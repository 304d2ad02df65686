"""Host part of the round's commit: cut each request's committed tokens where the per-token finish loop would stop.

Same rules and names as the reference's dependency-free ``selfspec_commit_rules.py``
(``patches/sglang/python/sglang/srt/speculative/selfspec_commit_rules.py:94-170``): a round commits
T = [a0] + the verified tokens (v[0..acc]); for a "fast" request (no grammar, no stop strings / regexes, no pending
abort) the per-token loop's first stop is

    j = min(budget - 1, first stop-set id, first out-of-vocab id, len(T) - 1),  budget = max_new_tokens - len(output)

and T[:j+1] is appended with one finish check.  Requests with a grammar or stop strings take the per-token loop
(``commit_slow``).  Works on any object with the SGLang ``Req`` attributes it reads (duck typed), and on the
lightweight ``Request`` of ``gravityocr_b200.compat``.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

_abort_reason_factory: Optional[Callable[[str], object]] = None


def set_abort_reason_factory(fn: Callable[[str], object]) -> None:
    global _abort_reason_factory
    _abort_reason_factory = fn


def grammar_accept_or_abort(req, token: int) -> bool:
    """Feed one committed token to the request's grammar; a rejection aborts the request (as AR decode does)."""
    try:
        req.grammar.accept_token(token)
        return True
    except ValueError:
        if _abort_reason_factory is None:
            raise
        req.to_finish = _abort_reason_factory(f"grammar rejected token {token}")
        req.check_finished()
        return False


def stop_set(req) -> frozenset:
    """Ids that finish the request (empty with ignore_eos); cached on the request."""
    s = getattr(req, "_ss_stop", None)
    if s is None:
        sp = req.sampling_params
        ids = set()
        if not sp.ignore_eos:
            ids |= set(sp.stop_token_ids or ())
            ids |= set(getattr(req, "eos_token_ids", None) or ())
            tk = getattr(req, "tokenizer", None)
            if tk is not None:
                if getattr(tk, "eos_token_id", None) is not None:
                    ids.add(tk.eos_token_id)
                ids |= set(getattr(tk, "additional_stop_token_ids", None) or ())
        s = frozenset(ids)
        req._ss_stop = s
    return s


def is_fast(req) -> bool:
    sp = req.sampling_params
    return (getattr(req, "grammar", None) is None and not getattr(req, "to_finish", None) and not req.finished()
            and not getattr(sp, "stop_strs", None) and not getattr(sp, "stop_regex_strs", None)
            and req.vocab_size is not None)


def cut_index(T: Sequence[int], budget: int, stop: frozenset, vocab: int) -> int:
    lim = len(T) - 1
    if budget - 1 < lim:
        lim = budget - 1 if budget > 0 else 0
    for t in range(lim):
        x = T[t]
        if x in stop or x > vocab or x < 0:
            return t
    return lim


def cannot_finish(req, T: Sequence[int]) -> bool:
    """True iff committing all of T leaves a fast request unfinished (host-only pre-check)."""
    if not is_fast(req):
        return False
    if req.sampling_params.max_new_tokens - len(req.output_ids) <= len(T):
        return False
    s = stop_set(req)
    if s and not s.isdisjoint(T):
        return False
    return min(T) >= 0 and max(T) <= req.vocab_size


def commit_fast(req, T: Sequence[int]) -> int:
    j = cut_index(T, req.sampling_params.max_new_tokens - len(req.output_ids), stop_set(req), req.vocab_size)
    req.output_ids.extend(T[: j + 1])
    req.check_finished(j + 1)
    return j


def commit_slow(req, T: Sequence[int]) -> Tuple[int, bool]:
    req.output_ids.append(T[0])
    req.check_finished()
    if req.finished():
        return 0, True
    if getattr(req, "grammar", None) is not None and not grammar_accept_or_abort(req, T[0]):
        return 0, True
    for t in range(1, len(T)):
        req.output_ids.append(T[t])
        req.check_finished()
        if req.finished():
            return t, False
        if getattr(req, "grammar", None) is not None and not grammar_accept_or_abort(req, T[t]):
            return t, False
    if getattr(req, "grammar", None) is not None and not req.finished():
        req.check_finished()
    return len(T) - 1, False


def host_commit(reqs, rows: Sequence[Sequence[int]]) -> Tuple[List[List[int]], List[int], List[int]]:
    """Apply packed rows (a0, acc, v[0..acc], zeros) to the requests.  Returns (tokens, j, acc) per request."""
    toks, js, accs = [], [], []
    for req, r in zip(reqs, rows):
        a = int(r[1])
        T = [int(r[0])] + [int(x) for x in r[2: 3 + a]]
        if is_fast(req):
            j = commit_fast(req, T)
            a0_fin = j == 0 and req.finished()
        else:
            j, a0_fin = commit_slow(req, T)
        req.spec_verify_ct = getattr(req, "spec_verify_ct", 0) + 1
        adt = 0 if a0_fin else a + 1
        req.spec_accepted_tokens = getattr(req, "spec_accepted_tokens", 0) + adt
        upd = getattr(req, "update_spec_acceptance_histogram", None)
        if upd is not None:
            upd(adt)
        toks.append(T[: j + 1])
        js.append(j)
        accs.append(a)
    return toks, js, accs
