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


def test_e4m3_decode_matches_cutlass():
    ref = load("mx_dec_e4m3.f32")
    lib = O.lib()
    got = np.array([lib.bho_e4m3_to_float(c) for c in range(256)], dtype=np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(nan, np.isnan(got)) and nan[0x7F] and nan[0xFF] and nan.sum() == 2
    assert np.array_equal(ref[~nan].view(np.uint32), got[~nan].view(np.uint32))


def test_e4m3_encode_matches_cutlass_on_every_bf16_pattern_and_tie():
    xs = load("mx_e4m3_in.f32")
    ref = load("mx_e4m3_out.u8")
    lib = O.lib()
    got = np.array([lib.bho_e4m3_from_float(float(x)) for x in xs], dtype=np.uint8)
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first: {xs[bad[:5]]} -> {got[bad[:5]]} vs {ref[bad[:5]]}"


def test_mxfp8_quantiser_follows_the_ocp_rule():
    rows, K = 8, 256
    X = O.gen_normal(19, rows * K).reshape(rows, K) * 5.0
    X[0, :32] = 0.0                     # all-zero block: code 0, zero elements
    X[1, :32] = 448.0                   # amax 448: exponent floor(log2 448) - 8 = 0
    X[1, 32:64] = 1.9 * 2.0 ** 8        # scaled amax 486.4 > 448: saturates to 448
    X[2, 5] = 1e-39                     # a subnormal inside a normal block
    q, sf = O.quantize_mxfp8(X)
    lib = O.lib()
    for r in range(rows):
        for b in range(K // 32):
            blk = X[r, b * 32:(b + 1) * 32]
            amax = float(np.max(np.abs(blk)))
            code = int(sf[O.sf_offset_vs(r, b, K, 32)])
            if amax < 2.0 ** -126:
                assert code == 0 and not q[r * K + b * 32:r * K + b * 32 + 32].any()
                continue
            e = int(np.floor(np.log2(amax))) - 8
            assert code == e + 127
            for i in range(32):
                want = lib.bho_e4m3_from_float(np.float32(blk[i] * np.float32(2.0 ** -e)))
                assert q[r * K + b * 32 + i] == want
    assert sf[O.sf_offset_vs(1, 0, K, 32)] == 127 and q[K] == 0x7E
    assert sf[O.sf_offset_vs(1, 1, K, 32)] == 127 and q[K + 32] == 0x7E   # saturated


def test_mixed_reference_gemm_dequantises_each_operand_in_its_format():
    M, N, K = 3, 5, 96
    xa = O.gen_normal(3, M * K).reshape(M, K) * 4.0
    xb = O.gen_normal(4, N * K).reshape(N, K)
    A, SFA = O.quantize_mxfp8(xa)
    B, SFB = O.quantize_mxfp4(xb)
    D, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, 1.0, fmt="mxf8f4")
    lib = O.lib()
    for m in range(M):
        a = [lib.bho_e4m3_to_float(int(A[m * K + k])) *
             lib.bho_ue8m0_to_float(int(SFA[O.sf_offset_vs(m, k // 32, K, 32)])) for k in range(K)]
        for n in range(N):
            acc = np.float32(0.0)
            for k in range(K):
                byte = int(B[(n * K + k) // 2])
                code = (byte >> 4) if k % 2 else (byte & 0xF)
                b = lib.bho_e2m1_to_float(code) * lib.bho_ue8m0_to_float(
                    int(SFB[O.sf_offset_vs(n, k // 32, K, 32)]))
                acc = np.float32(acc + np.float32(np.float32(a[k]) * np.float32(b)))
            assert D[m, n] == lib.bho_bf16_from_float(acc)
