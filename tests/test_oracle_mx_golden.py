"""The oracle's MXFP4 parts (UE8M0 decode, 128x4 layout with 32-element K groups, quantiser)
checked against CUTLASS 4.5.0's own host code (tests/golden/make_golden_mx.cpp) and against the
OCP MX v1.0 scaling rule."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    man = json.load(open(os.path.join(GOLD, "manifest_mx.json")))
    return np.fromfile(os.path.join(GOLD, name), dtype=man[name]["dtype"])


def test_ue8m0_decode_matches_cutlass():
    ref = load("mx_dec_ue8m0.f32")
    got = np.array([O.lib().bho_ue8m0_to_float(c) for c in range(256)], dtype=np.float32)
    assert np.isnan(ref[255]) and np.isnan(got[255])
    assert np.array_equal(ref[:255].view(np.uint32), got[:255].view(np.uint32))


@pytest.mark.parametrize("mn,k", [(128, 256), (256, 512), (200, 768), (16, 1024), (130, 320),
                                  (1, 128)])
def test_mx_sf_layout_matches_cutlass(mn, k):
    g = load(f"mx_sf_{mn}x{k}.i64")
    assert g[0] == g[1] == O.sf_storage_bytes_vs(mn, k, 32)
    offs = g[2:].reshape(mn, k // 32)
    for m in range(mn):
        for kg in range(k // 32):
            assert O.sf_offset_vs(m, kg, k, 32) == offs[m, kg]


def test_mx_layout_with_16_element_groups_is_the_nvfp4_layout():
    for mn, k in [(256, 512), (130, 320)]:
        assert O.sf_storage_bytes_vs(mn, k, 16) == O.sf_storage_bytes(mn, k)
        for m in (0, 1, 31, 32, 127, 128, mn - 1):
            for kg in (0, 1, 3, 4, k // 16 - 1):
                assert O.sf_offset_vs(m, kg, k, 16) == O.sf_offset(m, kg, k)


def test_mxfp4_quantiser_follows_the_ocp_rule():
    rows, K = 8, 256
    X = O.gen_normal(9, rows * K).reshape(rows, K) * 3.0
    X[0, :32] = 0.0                     # an all-zero block
    X[1, :32] = 6.0                     # amax exactly 6: exponent floor(log2 6) - 2 = 0
    X[2, 5] = 1e-39                     # a subnormal inside an otherwise normal block
    packed, sf = O.quantize_mxfp4(X)
    lib = O.lib()
    for r in range(rows):
        for b in range(K // 32):
            blk = X[r, b * 32:(b + 1) * 32]
            amax = float(np.max(np.abs(blk)))
            code = int(sf[O.sf_offset_vs(r, b, K, 32)])
            if amax < 2.0 ** -126:
                assert code == 0
                continue
            e = int(np.floor(np.log2(amax))) - 2
            assert code == e + 127
            for i in range(32):
                byte = packed[(r * K + b * 32 + i) // 2]
                q = (byte >> 4) if i % 2 else (byte & 0xF)
                assert q == lib.bho_e2m1_from_float(np.float32(blk[i] * np.float32(2.0 ** -e)))
    # dequantised values stay within one e2m1 step of the inputs (saturation at 6 * 2^e)
    assert sf[O.sf_offset_vs(1, 0, K, 32)] == 127


def test_mx_reference_gemm_uses_the_mx_scales():
    M, N, K = 4, 8, 128
    xa = O.gen_normal(1, M * K).reshape(M, K)
    xb = O.gen_normal(2, N * K).reshape(N, K)
    A, SFA = O.quantize_mxfp4(xa)
    B, SFB = O.quantize_mxfp4(xb)
    D, _ = O.gemm_full(M, N, K, A, SFA, B, SFB, 1.0, fmt="mxfp4")
    lib = O.lib()

    def deq(P, SF, rows):
        out = np.zeros((rows, K), dtype=np.float64)
        for r in range(rows):
            for k in range(K):
                byte = P[(r * K + k) // 2]
                q = (byte >> 4) if k % 2 else (byte & 0xF)
                s = lib.bho_ue8m0_to_float(int(SF[O.sf_offset_vs(r, k // 32, K, 32)]))
                out[r, k] = lib.bho_e2m1_to_float(int(q)) * s
        return out

    ref = deq(A, SFA, M) @ deq(B, SFB, N).T
    got = O.bf16_bits_to_f32(D)
    assert np.allclose(got, ref, rtol=2 ** -7, atol=1e-30)
