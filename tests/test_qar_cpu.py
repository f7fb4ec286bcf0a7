"""Host-side parts of the compressed all-reduce: the knob and the CPU statement of the math."""
import pytest
import torch

from vllm_suffix_hybrid_b200.parallel.symm import qar_mode, qar_reference


def test_qar_mode_names():
    assert qar_mode("") == 0 and qar_mode("off") == 0 and qar_mode(None) == 0
    assert qar_mode("int8") == 1 and qar_mode("FP8") == 2
    with pytest.raises(ValueError):
        qar_mode("int4")


@pytest.mark.parametrize("mode,rel", [(1, 1 / 254), (2, 1 / 16)])
@pytest.mark.parametrize("two_shot", [False, True])
def test_reference_error_within_block_bound(mode, rel, two_shot):
    """Every decoded value is within half a code step of its input (int8: amax / 254 per block; e4m3: 1/16
    of the value plus a subnormal step), so the sum of W contributions is within W such steps (plus one
    more for the requantised gather of the two-shot form)."""
    g = torch.Generator().manual_seed(mode + 2 * two_shot)
    world, T, H = 4, 8, 1024
    parts = [torch.randn(T, H, generator=g) * (1 + 10 * torch.rand(T, 1, generator=g)) for _ in range(world)]
    parts[0][:, 5] = 300.0  # an outlier channel: its blocks get a coarse scale
    got = qar_reference(parts, mode, two_shot)
    exact = sum(parts)

    def amax(x):
        return x.view(T, H // 128, 128).abs().amax(-1, keepdim=True).expand(T, H // 128, 128).reshape(T, H)

    if mode == 1:
        bound = sum(amax(p) * rel for p in parts)
        if two_shot:
            bound = bound + amax(exact.abs() + bound) * rel
    else:
        bound = sum(p.abs() * rel + amax(p) / 448 / 512 for p in parts)
        if two_shot:
            bound = bound + (exact.abs() + bound) * rel + amax(exact.abs() + bound) / 448 / 512
    assert bool(((got - exact).abs() <= bound * 1.0001 + 1e-6).all())


def test_reference_is_order_fixed_and_zero_safe():
    parts = [torch.zeros(2, 256), torch.ones(2, 256)]
    a = qar_reference(parts, 1)
    b = qar_reference([p.clone() for p in parts], 1)
    assert torch.equal(a, b)
    assert torch.equal(qar_reference([torch.zeros(3, 128)], 2, True), torch.zeros(3, 128))
