"""The advisory host-array GEMM crossover (choose_gemm_backend, the rule of
packages/tensor-webgpu/src/threshold.ts:67-85 with this device's measured thresholds) on the CPU."""
import pytest

from tensor_cuda.caps import GEMM_ELEMENT_THRESHOLD, GEMM_WORK_THRESHOLD, chooseGemmBackend, choose_gemm_backend


def test_rule_shape_follows_the_reference():
    e, w = GEMM_ELEMENT_THRESHOLD, GEMM_WORK_THRESHOLD
    # below the element threshold: CPU whatever k is
    assert choose_gemm_backend(1, e - 1, 1 << 20) == "cpu"
    # at the element threshold: the work test decides when k is given
    k_small = max(0, w // e - 1)
    assert choose_gemm_backend(1, e, k_small) == ("cpu" if e * k_small < w else "cuda")
    assert choose_gemm_backend(1, e, -(-w // e)) == "cuda"
    # k omitted: only the element test applies (the reference's (m, n) signature)
    assert choose_gemm_backend(1, e) == "cuda"
    assert chooseGemmBackend is choose_gemm_backend


def test_large_products_go_to_the_device_and_tiny_ones_stay():
    assert choose_gemm_backend(2048, 2048, 2048) == "cuda"
    assert choose_gemm_backend(4, 4, 4) == "cpu"


@pytest.mark.parametrize("bad", [(-1, 4, 4), (4, 4.5, 4), (4, 4, -2)])
def test_rejects_bad_sizes(bad):
    with pytest.raises(ValueError):
        choose_gemm_backend(*bad)
