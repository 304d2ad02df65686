"""Host-side attention planning (no GPU): the split plan that both attention kernels are launched with."""
import math

import pytest

from gravityocr_b200.engine import attention_split

SMS = 148


@pytest.mark.parametrize("bs", [1, 2, 3, 8, 16, 17, 18, 36, 37, 64, 128])
@pytest.mark.parametrize("max_len", [16, 300, 1024, 2770, 4128, 8192, 16384])
def test_split_plan_invariants(bs, max_len):
    """Chunks are whole 64-token tiles of at most 4096 tokens (the kernels' page-id buffer), the splits cover every
    visible position including the window, there are at most 16 of them (the merges' limit) and at most 8 when the
    grid is smaller than two CTAs per SM (those splits are merged inside one portable thread-block cluster)."""
    K, n_kv = 17, 8
    chunk, splits = attention_split(bs, K, max_len, max_len, n_kv, SMS)
    L = max_len + K + 1
    assert chunk % 64 == 0 and 64 <= chunk <= 4096
    assert splits == math.ceil(L / chunk) and chunk * splits >= L
    assert splits <= 16
    if bs * n_kv < 2 * SMS:
        assert splits <= 8


def test_large_batches_are_unsplit_below_one_chunk():
    """With two CTAs per SM already filled by (request, kv head) pairs, requests shorter than a chunk run unsplit."""
    chunk, splits = attention_split(64, 17, 4000, 2200, 8, SMS)
    assert (chunk, splits) == (4096, 1)


def test_small_batches_split_for_parallelism():
    """A single request is cut into splits of >= 128 tokens so that its CTAs stream in parallel."""
    chunk, splits = attention_split(1, 17, 2770, 2770, 8, SMS)
    assert chunk >= 128 and 2 <= splits <= 8
