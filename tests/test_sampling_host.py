"""Host side of the non-greedy round (no GPU): request normalisation, the plain-batch test, the filter the batch
block selects, and the grammar bit packing."""
import torch

from gravityocr_b200 import _lib as L
from gravityocr_b200.sampling import TOP_K_ALL, RequestSampling, SamplerState, pack_allowed


def test_normalisation_follows_sglang_sampling_params():
    # temperature below 1e-6 is greedy (temperature 1, top_k 1); top_k <= 0 keeps every token
    assert RequestSampling(temperature=0.0).normalised() == (1.0, 1)
    assert RequestSampling(temperature=0.7, top_k=-1).normalised() == (0.7, TOP_K_ALL)
    assert RequestSampling(temperature=0.0).plain
    assert not RequestSampling(temperature=0.0, repetition_penalty=1.1).plain
    assert not RequestSampling(temperature=0.5).plain


def test_flashinfer_batch_with_min_p_takes_the_sequential_filter():
    """selfspec_sampling.verify_target_probs: the flashinfer backend renormalises by top-k, then top-p, then applies
    min-p as soon as one request of the batch sets min_p; without min-p it keeps the joint rule."""
    st = SamplerState(64, 4, "cpu", filter=L.FILTER_JOINT)
    rpi = torch.arange(2, dtype=torch.int64)
    plain = [RequestSampling(temperature=0.8, top_p=0.9)] * 2
    assert st.batch(plain, rpi).filter == L.FILTER_JOINT
    mixed = [RequestSampling(temperature=0.8, top_p=0.9), RequestSampling(temperature=0.8, min_p=0.05)]
    assert st.batch(mixed, rpi).filter == L.FILTER_SEQUENTIAL
    st_torch = SamplerState(64, 4, "cpu", filter=L.FILTER_TORCH)
    assert st_torch.batch(mixed, rpi).filter == L.FILTER_TORCH


def test_penalizer_order_keeps_only_used_penalizers():
    st = SamplerState(64, 4, "cpu")
    rpi = torch.arange(2, dtype=torch.int64)
    s = st.batch([RequestSampling(temperature=1.0, repetition_penalty=1.2),
                  RequestSampling(temperature=1.0, frequency_penalty=0.3)], rpi)
    assert list(s.order[: s.n_order]) == [L.PEN_FREQUENCY, L.PEN_REPETITION]


def test_pack_allowed_bit_layout():
    allowed = torch.zeros((2, 70), dtype=torch.bool)
    allowed[0, [0, 31, 32, 69]] = True
    allowed[1, 5] = True
    bits = pack_allowed(allowed)
    assert bits.shape == (2, 3) and bits.dtype == torch.int32
    w = bits.view(torch.int32).tolist()
    assert w[0][0] & 1 and (w[0][0] >> 31) & 1 and w[0][1] & 1 and (w[0][2] >> 5) & 1
    assert w[1] == [1 << 5, 0, 0]
