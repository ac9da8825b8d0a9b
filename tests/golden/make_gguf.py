"""Writes tests/golden/tiny_ptq.gguf with the reference's own GGUF writer
(bd::GgufWriter, ref/bonsai-decoder/include/bd/gguf.hpp:88-114, compiled into
oracle/_ref/libbtf_ref.so) and records its checksum and each tensor's data
offset as the reference's reader (bd::Gguf) reports it in MANIFEST_GGUF.json.

Tensors: two seeded PTQ1_0 matrices (type 143, ne0 = K columns, ne1 = N rows)
of ragged shapes and one small f32 vector; metadata of several value kinds.
Run: python tests/golden/make_gguf.py
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "bonsai-ternary-fast_b200"))

PTQ1_0 = 143
F32 = 0
TENSORS = [("blk.0.ffn_up.weight", 1152, 37, PTQ1_0, 51), ("blk.0.attn_q.weight", 2048, 16, PTQ1_0, 52),
           ("output_norm.weight", 64, 1, F32, 53)]


def main():
    import oracle
    import synth

    if not oracle.Reference.available():
        raise SystemExit("oracle/_ref/libbtf_ref.so is missing: run `make -C oracle` where the reference tree exists")
    L = oracle.Reference().L
    L.ref_gguf_write.restype = ctypes.c_int
    L.ref_gguf_tensor_offset.restype = ctypes.c_int64
    L.ref_gguf_tensor_offset.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
    blobs = []
    for name, K, N, typ, seed in TENSORS:
        if typ == PTQ1_0:
            blobs.append(np.ascontiguousarray(synth.ternary_ptq(N, K, seed=seed)).reshape(-1))
        else:
            blobs.append(np.random.default_rng(seed).standard_normal(K * N).astype(np.float32).view(np.uint8))
    n = len(TENSORS)
    names = (ctypes.c_char_p * n)(*[t[0].encode() for t in TENSORS])
    ne0 = (ctypes.c_int64 * n)(*[t[1] for t in TENSORS])
    ne1 = (ctypes.c_int64 * n)(*[t[2] for t in TENSORS])
    types = (ctypes.c_uint32 * n)(*[t[3] for t in TENSORS])
    data = (ctypes.c_void_p * n)(*[b.ctypes.data for b in blobs])
    nbytes = (ctypes.c_uint64 * n)(*[b.size for b in blobs])
    path = os.path.join(HERE, "tiny_ptq.gguf")
    rc = L.ref_gguf_write(path.encode(), n, names, ne0, ne1, types, data, nbytes, 32)
    if rc:
        raise SystemExit(f"ref_gguf_write failed ({rc})")
    meta = {"file": "tiny_ptq.gguf", "sha256": hashlib.sha256(open(path, "rb").read()).hexdigest(), "tensors": []}
    for (name, K, N, typ, seed), b in zip(TENSORS, blobs):
        meta["tensors"].append({"name": name, "ne0": K, "ne1": N, "type": typ, "seed": seed, "bytes": int(b.size),
                                "file_offset": int(L.ref_gguf_tensor_offset(path.encode(), name.encode())),
                                "sha256": hashlib.sha256(b.tobytes()).hexdigest()})
    with open(os.path.join(HERE, "MANIFEST_GGUF.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
