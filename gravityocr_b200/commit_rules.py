"""Host part of the round's commit: how many of a round's committed tokens each request keeps.

A round commits T = [a0] + v[0..acc] for a request.  SGLang appends decode tokens one at a time and checks the finish
conditions after each; the served worker must end a request exactly where that loop would.  The contract restated
here is the one of the reference's ``selfspec_commit_rules.py`` (``patches/sglang/python/sglang/srt/speculative/
selfspec_commit_rules.py:94-170``; the function names are kept because the worker hooks and tests use them):

  * a request is *plain* when nothing but its length budget and a set of stop ids can end it: no grammar, no pending
    abort, not finished, no stop strings or regexes, a known vocabulary size.  For a plain request the loop's stopping
    point is known from T alone: the index
        j = min(budget - 1, first index holding a stop id or an id outside [0, vocab], len(T) - 1)
    where budget = max_new_tokens - len(output_ids) (a budget of 0 or less still appends one token).  T[:j+1] is
    appended and the finish check runs once over those tokens.
  * any other request walks T token by token: append, check, feed its grammar (a grammar rejection aborts the request
    through ``set_abort_reason_factory``), stop at the first finish.
  * the acceptance counters advance by acc + 1 per round, except when a0 alone ended the request (then 0).

``oracle/commit_ref.py`` and the golden vectors made from the reference module pin these rules in the tests.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

_abort_reason_factory: Optional[Callable[[str], object]] = None


def set_abort_reason_factory(fn: Callable[[str], object]) -> None:
    """How a grammar rejection becomes the request's finish reason (the serving framework's abort type)."""
    global _abort_reason_factory
    _abort_reason_factory = fn


def grammar_accept_or_abort(req, token: int) -> bool:
    """Feed one committed token to the request's grammar; False (and the request aborted) when it is rejected."""
    try:
        req.grammar.accept_token(token)
    except ValueError:
        if _abort_reason_factory is None:
            raise
        req.to_finish = _abort_reason_factory(f"grammar rejected token {token}")
        req.check_finished()
        return False
    return True


def stop_set(req) -> frozenset:
    """Token ids that end the request: its stop ids, its EOS ids and its tokenizer's; none under ignore_eos.
    Computed once per request."""
    cached = getattr(req, "_ss_stop", None)
    if cached is not None:
        return cached
    sp = req.sampling_params
    ids: set = set()
    if not sp.ignore_eos:
        ids.update(sp.stop_token_ids or ())
        ids.update(getattr(req, "eos_token_ids", None) or ())
        tk = getattr(req, "tokenizer", None)
        if tk is not None:
            if getattr(tk, "eos_token_id", None) is not None:
                ids.add(tk.eos_token_id)
            ids.update(getattr(tk, "additional_stop_token_ids", None) or ())
    req._ss_stop = frozenset(ids)
    return req._ss_stop


def is_fast(req) -> bool:
    """A plain request (see the module docstring): its cut follows from the tokens alone."""
    sp = req.sampling_params
    blocked = (getattr(req, "grammar", None) is not None, bool(getattr(req, "to_finish", None)), req.finished(),
               bool(getattr(sp, "stop_strs", None)), bool(getattr(sp, "stop_regex_strs", None)),
               req.vocab_size is None)
    return not any(blocked)


def _ends(t: int, stop: frozenset, vocab: int) -> bool:
    return t in stop or t < 0 or t > vocab


def cut_index(T: Sequence[int], budget: int, stop: frozenset, vocab: int) -> int:
    """Index of the last token a plain request keeps from T."""
    last = min(len(T) - 1, max(budget - 1, 0))
    return next((i for i in range(last) if _ends(T[i], stop, vocab)), last)


def cannot_finish(req, T: Sequence[int]) -> bool:
    """True iff appending all of T certainly leaves a plain request running (budget left, no stop or bad id)."""
    if not is_fast(req) or req.sampling_params.max_new_tokens - len(req.output_ids) <= len(T):
        return False
    stop = stop_set(req)
    return not any(_ends(t, stop, req.vocab_size) for t in T)


def commit_fast(req, T: Sequence[int]) -> int:
    """Plain request: append T[:j+1] with one finish check; returns j."""
    j = cut_index(T, req.sampling_params.max_new_tokens - len(req.output_ids), stop_set(req), req.vocab_size)
    req.output_ids.extend(T[: j + 1])
    req.check_finished(j + 1)
    return j


def commit_slow(req, T: Sequence[int]) -> Tuple[int, bool]:
    """Any request: the per-token loop.  Returns (index of the last token kept, whether a0 alone ended it)."""
    has_grammar = getattr(req, "grammar", None) is not None
    for i, t in enumerate(T):
        req.output_ids.append(t)
        req.check_finished()
        if req.finished():
            return i, i == 0
        if has_grammar and not grammar_accept_or_abort(req, t):
            return i, i == 0
    if has_grammar and not req.finished():
        req.check_finished()
    return len(T) - 1, False


def host_commit(reqs, rows: Sequence[Sequence[int]]) -> Tuple[List[List[int]], List[int], List[int]]:
    """Apply the round's packed rows (a0, acc, v[0..acc], zeros...) to the requests.  Returns the kept tokens, j and
    acc of each request."""
    toks: List[List[int]] = []
    js: List[int] = []
    accs: List[int] = []
    for req, row in zip(reqs, rows):
        acc = int(row[1])
        T = [int(row[0])] + [int(t) for t in row[2: 3 + acc]]
        if is_fast(req):
            j = commit_fast(req, T)
            a0_only = j == 0 and req.finished()
        else:
            j, a0_only = commit_slow(req, T)
        gained = 0 if a0_only else acc + 1
        req.spec_verify_ct = getattr(req, "spec_verify_ct", 0) + 1
        req.spec_accepted_tokens = getattr(req, "spec_accepted_tokens", 0) + gained
        hist = getattr(req, "update_spec_acceptance_histogram", None)
        if hist is not None:
            hist(gained)
        toks.append(T[: j + 1])
        js.append(j)
        accs.append(acc)
    return toks, js, accs
