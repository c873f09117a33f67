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
