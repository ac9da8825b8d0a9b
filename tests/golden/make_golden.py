"""Generates the golden fixtures of tests/golden/ from the reference's OWN code.

The reference keeps no stored numeric vectors (its tests generate inputs in
the test body: tests/test_packed.cpp, tests/test_gpu_kernels.cpp), so these
fixtures are made here, once, by the reference's C++ compiled from its sources
(oracle/_ref/libbtf_ref.so, built by oracle/Makefile where the reference tree
is present) and committed with this script:

  src      PTQ1_0 blocks, encoded by bd::quant_row (ref/bonsai-decoder/src/types.cpp:289-320)
  codes,   T2 codes / fp16 scales from btf::repack_rows (src/repack.cpp:16-27)
  scales
  q, d, s  Q8_0 of x from btf::q8_block_host (include/btf/packed.hpp:117-134)
  idot     btf::sub_dot_host (include/btf/packed.hpp:108-113) minus s, per (m, row, sub-block)
  y_store  the emulator GEMV loop (src/emu_decoder.cpp:143-165), y = W x
  y_add    the same with add: y = y0 + W x
  up_*     a second matrix of the same shape (the "up" half of a swiglu pair)

Inputs are seeded: trits uniform over {-1, 0, 1}, block scales fp16(|N(0,1)| * 0.02),
x ~ N(0, 1) with planted edge blocks (all-zero, tiny, large, all-negative).
Run: python tests/golden/make_golden.py  (writes *.npz and MANIFEST.json here).
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "bonsai-ternary-fast_b200"))

# name: (N, K, M, seed)
CASES = {
    "small": (24, 256, 2, 11),
    "ragged": (37, 1152, 3, 21),
    "wide": (16, 5120, 1, 31),
}


def _inputs(N, K, M, seed):
    rng = np.random.default_rng(seed)
    t = rng.integers(-1, 2, size=(N, K)).astype(np.int8)
    sc = np.abs(rng.standard_normal((N, K // 128))) * 0.02
    sc16 = sc.astype(np.float16).astype(np.float32)
    w = t.astype(np.float32) * np.repeat(sc16, 128, axis=1)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[0, 32:64] = 0.0                                    # all-zero block: d = 0, q = 0
    if M > 1:
        x[1, 64:96] *= 1e-30                             # tiny block
        x[1, 96:128] = -np.abs(x[1, 96:128])             # all-negative block
    if M > 2:
        x[2, 0:32] *= 1e4                                # large block
    return w, t, sc16, x


def make_case(ref, N, K, M, seed):
    import synth

    w, t, sc16, x = _inputs(N, K, M, seed)
    src = ref.ptq_quant_rows(w)                          # the reference's encoder
    assert np.array_equal(src, synth.encode_ptq1_0(t, sc16.astype(np.float16).view(np.uint16))), "encoder mismatch"
    codes, scales = ref.repack_rows(src, N, K)
    q, d, s = ref.q8_rows(x)
    idot = np.empty((M, N, K // 32), dtype=np.int32)
    aw = q.view(np.uint32).reshape(M, K // 4)
    cw = codes.view(np.uint32).reshape(N, K // 16)
    for m in range(M):
        for n in range(N):
            for b in range(K // 32):
                a8 = np.ascontiguousarray(aw[m, 8 * b:8 * b + 8])
                idot[m, n, b] = ref.L.ref_sub_dot(int(cw[n, 2 * b]), int(cw[n, 2 * b + 1]), a8.ctypes.data) - s[m, b]
    y_store = ref.gemv(codes, scales, K, q, d, s)
    y0 = np.random.default_rng(seed + 1).standard_normal((M, N)).astype(np.float32)
    y_add = ref.gemv(codes, scales, K, q, d, s, y=y0.copy(), add=True)
    # second matrix (swiglu "up")
    w2, t2, sc2, _ = _inputs(N, K, M, seed + 100)
    up_src = ref.ptq_quant_rows(w2)
    up_codes, up_scales = ref.repack_rows(up_src, N, K)
    up_y = ref.gemv(up_codes, up_scales, K, q, d, s)
    return dict(N=N, K=K, M=M, src=src, x=x, codes=codes, scales=scales, q=q, d=d, s=s, idot=idot,
                y_store=y_store, y0=y0, y_add=y_add, up_src=up_src, up_codes=up_codes, up_scales=up_scales,
                up_y=up_y)


def main():
    import oracle

    if not oracle.Reference.available():
        raise SystemExit("oracle/_ref/libbtf_ref.so is missing: run `make -C oracle` where the reference tree exists")
    ref = oracle.Reference()
    manifest = {"generator": "tests/golden/make_golden.py", "cases": {}}
    for name, (N, K, M, seed) in CASES.items():
        arrays = make_case(ref, N, K, M, seed)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        manifest["cases"][name] = {"N": N, "K": K, "M": M, "seed": seed,
                                   "sha256": hashlib.sha256(open(path, "rb").read()).hexdigest()}
        print(name, N, K, M, os.path.getsize(path), "bytes")
    with open(os.path.join(HERE, "MANIFEST.json"), "w") as f:
        json.dump(manifest, f, indent=1)


if __name__ == "__main__":
    main()
