"""The projection planner (no GPU: the library plans for 148 SMs when no device is present), through gr_linear_plan:
every plan covers its rows with whole MMA-shaped tiles and a split count that divides K, and the plans the decoder's
projections get at the benchmarked sizes are the measured ones."""
import pytest

from gravityocr_b200 import _lib as L

SHAPES = [(4096, 1536, L.EPI_QKV_ROPE), (1536, 2048, L.EPI_PARTIAL_F32), (9216, 1536, L.EPI_SWIGLU),
          (1536, 4608, L.EPI_PARTIAL_F32), (59392, 1536, L.EPI_ARGMAX), (59392, 1536, L.EPI_STORE_F32)]


@pytest.mark.parametrize("n_out,k_in,mode", SHAPES)
@pytest.mark.parametrize("m", [1, 5, 17, 34, 68, 136, 272, 408, 544, 816, 1088, 1632, 2176, 4224])
def test_plan_invariants(n_out, k_in, mode, m):
    p = L.linear_plan(n_out, k_in, m, mode)
    assert p["splits"] == L.linear_default_splits(n_out, k_in, m, mode)
    assert (k_in // 64) % p["splits"] == 0
    assert p["nt"] % 16 == 0 and 16 <= p["nt"] <= 256
    assert p["m_tiles"] * p["nt"] >= m > (p["m_tiles"] - 1) * p["nt"]
    if p["m_tiles"] > 1:
        assert p["nt"] >= 128          # narrow multi-tile plans would re-read every weight tile
    if mode == L.EPI_ARGMAX:
        assert p["splits"] == 1
    units = (n_out // 128) * p["m_tiles"] * p["splits"]
    assert 1 <= p["grid"] <= min(units, 2 * 148)
    if p["tail_last"]:
        assert m % p["nt"] != 0 and n_out * k_in * 2 <= 48 << 20


def test_benchmarked_plans():
    """Config 3 (1,088 rows): QKV as four 256-row tiles and a 64-row tile numbered last (one wave), o_proj / down_proj
    as two splits of 192-row tiles; batch 1 (17 rows): one 32-row tile and split-K for every projection but lm_head."""
    qkv = L.linear_plan(4096, 1536, 1088, L.EPI_QKV_ROPE)
    assert (qkv["nt"], qkv["m_tiles"], qkv["splits"], qkv["tail_last"]) == (256, 5, 1, True)
    for k_in in (2048, 4608):
        p = L.linear_plan(1536, k_in, 1088, L.EPI_PARTIAL_F32)
        assert (p["nt"], p["m_tiles"], p["splits"]) == (192, 6, 2)
    for n_out, k_in, mode in SHAPES[:4]:
        p = L.linear_plan(n_out, k_in, 17, mode)
        assert (p["nt"], p["m_tiles"]) == (32, 1) and p["splits"] > 1
    assert L.linear_plan(59392, 1536, 17, L.EPI_ARGMAX)["splits"] == 1


def test_plan_rejects_bad_shapes():
    with pytest.raises(RuntimeError):
        L.linear_plan(1000, 1536, 17)           # n_out not a multiple of 128
    with pytest.raises(RuntimeError):
        L.linear_plan(4096, 1536, 17, L.EPI_STORE_F32, splits=5)   # 24 K chunks do not split in 5
