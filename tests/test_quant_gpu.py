"""GPU NVFP4 quantiser vs the oracle's host quantiser: bit-exact packed codes, scale
factors (padding included) and global scale, through the C ABI."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _run(x_np, bf16=False):
    import torch
    import blackhole_b200 as bh

    x = torch.from_numpy(x_np).cuda()
    if bf16:
        x = x.to(torch.bfloat16)
    rows, K = x.shape
    packed = torch.full((rows * K // 2,), 0xAB, dtype=torch.uint8, device="cuda")
    sf = torch.full((bh.sf_storage_bytes(rows, K),), 0xCD, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(2, dtype=torch.float32, device="cuda")
    bh.nvfp4_quantize(x, rows, K, packed, sf, scales, x_is_bf16=bf16)
    torch.cuda.synchronize()
    return packed.cpu().numpy(), sf.cpu().numpy(), scales.cpu().numpy()


@pytest.mark.parametrize("rows,K,std,outl", [(128, 256, 1.0, 0.0), (200, 768, 0.02, 0.0),
                                             (1, 4096, 1.0, 0.0), (333, 1024, 1.0, 0.01),
                                             (1024, 1024, 1.0, 0.0), (16, 80, 3.0, 0.0)])
def test_quantizer_bit_exact_f32(rows, K, std, outl):
    x = O.gen_normal(rows * 31 + K, rows * K, 0.0, std).reshape(rows, K)
    if outl:
        O.apply_outliers(9, x.reshape(-1), outl, 20.0)
    p_ref, sf_ref, g_ref = O.quantize(x)
    p, sf, sc = _run(x)
    assert sc[0] == np.abs(x).max()
    assert sc[1] == np.float32(g_ref)
    assert np.array_equal(p, p_ref)
    assert np.array_equal(sf, sf_ref)


def test_quantizer_bit_exact_bf16_input():
    import torch
    rows, K = 256, 512
    x = O.gen_normal(77, rows * K).reshape(rows, K)
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()  # the values the GPU sees
    p_ref, sf_ref, g_ref = O.quantize(xb)
    p, sf, sc = _run(x, bf16=True)
    assert sc[1] == np.float32(g_ref)
    assert np.array_equal(p, p_ref) and np.array_equal(sf, sf_ref)


def test_quantizer_all_zero_tensor():
    x = np.zeros((128, 256), np.float32)
    p, sf, sc = _run(x)
    assert sc[0] == 0 and sc[1] == 0
    assert not p.any() and not sf.any()


def _tie_matrix():
    """Blocks whose quotients sit exactly on rounding thresholds.  amax = 5.25 makes the global
    scale g = 5.25 / 2688 = 2^-9 exact; a block with amax 25.5 * 2^-9 has (amax/6)/g = 4.25, a
    UE4M3 midpoint (rounds to 4), so its scale is 4 * 2^-9 = 2^-7 and its elements t * 2^-7
    divide to exactly t, every E2M1 midpoint and its negative; other blocks do the same at the
    saturated scale 448 (scale 0.875) and put tiny values (codes 0 and negative 0) next to them."""
    mids = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    rows, K = 4, 64
    x = np.zeros((rows, K), np.float32)
    s7 = 2.0 ** -7
    x[0, :16] = [6.375 * s7] + [t * s7 for t in mids] + [-t * s7 for t in mids] + [0.0]
    x[1, :16] = [5.25] + [t * 0.875 for t in mids] + [-t * 0.875 for t in mids] + [-1e-6]
    x[2, 16:32] = [25.5 * 2.0 ** -9] + [-0.01 * s7, 0.01 * s7, -0.0] + [(i - 6) * 0.3 * s7 for i in range(12)]
    x[3, :] = O.gen_normal(5, K, 0.0, 0.5)
    return x


def test_quantizer_ties_and_signed_zeros_bit_exact():
    x = _tie_matrix()
    p_ref, sf_ref, g_ref = O.quantize(x)
    assert g_ref == 2.0 ** -9
    p, sf, sc = _run(x)
    assert sc[1] == np.float32(g_ref)
    assert np.array_equal(sf, sf_ref)
    assert np.array_equal(p, p_ref), np.nonzero(p != p_ref)


def test_quantizer_large_ragged_bit_exact():
    """Many rows (several passes of the persistent grid), K not a multiple of 128 (partial
    last segments) and a row count that is not a multiple of 128 (padding rows)."""
    rows, K = 1500, 2000 - 2000 % 16 + 16
    x = O.gen_normal(123, rows * K, 0.0, 2.0).reshape(rows, K)
    p_ref, sf_ref, g_ref = O.quantize(x)
    p, sf, sc = _run(x)
    assert sc[1] == np.float32(g_ref)
    assert np.array_equal(sf, sf_ref) and np.array_equal(p, p_ref)
