"""Regenerate the golden vectors in tests/golden/ from the reference's own code.

    make -C oracle ref REF=<reference checkout>
    python tests/golden/make_golden.py

Every array comes from oracle/_ref/libk200ref.so, i.e. the reference's
bench/native-q4-reference.h, src/q4-layout.cpp and src/q4-common-pack.h
compiled where they lie, plus closed-form inputs of bench/library-bench.cpp
(restated, as the reference computes them inline in main()).  The CPU oracle
is then pinned against these files by tests/test_oracle_pins.py, which keeps
working on machines where the reference checkout is absent.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402


def ref_fixture(R, k, n):
    q4 = np.empty(n * k // 32 * 18, np.uint8)
    dec = np.empty(n * k, np.float32)
    nat = np.empty(((n + 31) // 32 * 32) * k // 2, np.uint8)
    rs = np.empty(n, np.float32)
    R.ref_fixture(k, n, q4.ctypes.data, dec.ctypes.data, nat.ctypes.data, rs.ctypes.data)
    return q4, dec, nat, rs


def main() -> None:
    R = O.ref()
    if R is None:
        raise SystemExit("oracle/_ref/libk200ref.so is not built (make -C oracle ref REF=...)")
    out = {}
    # 1. Weights fixture (xorshift seed 0x7340d123), its decode and the bench's
    #    own native packing, at a shape with an N tail and an odd block count.
    k, n = 96, 33
    q4, dec, nat, rs = ref_fixture(R, k, n)
    out["fx_q4_k96_n33"] = q4
    out["fx_decoded_k96_n33"] = dec
    out["fx_rowscale_k96_n33"] = rs
    size = R.ref_native_q4_size(k, n)
    packed = np.empty(size, np.uint8)
    assert R.ref_pack_native_q4(packed, size, q4, k, n) == 1
    out["native_k96_n33"] = packed
    # 2. Input fixtures, patterns 0..4 (seed 0x09200abc), K=256 batch 2.
    for pattern in range(5):
        x = np.empty(256 * 2, np.float32)
        R.ref_input(256, 2, pattern, x)
        out[f"input_k256_b2_p{pattern}"] = x
    # 3. Two-component A8 activation model (native_q4_bench::Activation) for
    #    pattern 0 and 1, K=256 batch 1.
    for pattern in (0, 1):
        x = np.empty(256, np.float32)
        R.ref_input(256, 1, pattern, x)
        lin = np.empty(2 * 256, np.int8)
        sc = np.empty(3, np.float32)
        rep = np.empty(256, np.float32)
        R.ref_activation(x, 256, 1, 8, 2, lin, sc, rep.ctypes.data)
        out[f"a8_linear_p{pattern}"] = lin
        out[f"a8_scales_p{pattern}"] = sc
        out[f"a8_represented_p{pattern}"] = rep
    # 4. FP64 reference() over the decoded fixture, K=256 N=65 batch 4.
    k, n, b = 256, 65, 4
    q4, dec, _, _ = ref_fixture(R, k, n)
    x = np.empty(k * b, np.float32)
    R.ref_input(k, b, 0, x)
    gold = np.empty(n * b, np.float64)
    R.ref_reference(dec, x, k, n, b, gold)
    out["fp64_q4_k256_n65"] = q4
    out["fp64_x_k256_b4"] = x
    out["fp64_gold_k256_n65_b4"] = gold
    # 5. Common Q4 ABI v1 pack (Micro32Bank, K-major) at an unpadded shape.
    k, n = 96, 33
    q4, _, _, _ = ref_fixture(R, k, n)
    info = (C.c_longlong * 6)()
    assert R.ref_common_pack(q4, q4.size, k, n, 1, 1, None, 0, info) == 1
    payload = np.empty(info[5], np.uint8)
    assert R.ref_common_pack(q4, q4.size, k, n, 1, 1, payload.ctypes.data, payload.size, info) == 1
    out["common_k96_n33"] = payload
    out["common_info_k96_n33"] = np.array(list(info), np.int64)
    np.savez_compressed(os.path.join(HERE, "reference_vectors.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
