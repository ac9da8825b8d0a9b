"""CPU restatement of the reference's batch-1 decode step — TEST INFRASTRUCTURE ONLY.

Restates btf::make_emu_decoder (src/emu_decoder.cpp of bonsai-ternary-fast,
`chunk` :167-220, `gdn` :222-303, `attn` :305-375) for one token per step over
a qwen35 GGUF, with the model binding of bd::Model::bind
(ref/bonsai-decoder/src/model.cpp:68-205). The matmul path reuses the plain-C
oracle (oracle.c: Q8_0, the T2 repack, the emulator GEMV loop and the prep,
each pinned bit-exact to the reference's own code); the rest is numpy float32
in the emulator's order, with the sums whose order matters taken sequentially
(cumsum). It is checked against the reference emulator itself
(tests/test_decoder_oracle.py) and is never linked by the product.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import struct

import numpy as np

# The emulator's float transcendentals are the C library's expf / log1pf /
# cosf / sinf / powf; numpy's own float32 kernels can differ in the last ulp,
# which a Q8 requantisation occasionally turns into a flipped int8 code.
_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
for _n in ("expf", "log1pf", "cosf", "sinf"):
    getattr(_libm, _n).restype, getattr(_libm, _n).argtypes = ctypes.c_float, [ctypes.c_float]
_libm.powf.restype, _libm.powf.argtypes = ctypes.c_float, [ctypes.c_float, ctypes.c_float]


def _vec1(name):
    f = getattr(_libm, name)
    u = np.frompyfunc(lambda v: f(float(v)), 1, 1)
    return lambda x: np.float32(f(float(x))) if np.ndim(x) == 0 else u(np.asarray(x, np.float32)).astype(np.float32)


expf, log1pf, cosf, sinf = _vec1("expf"), _vec1("log1pf"), _vec1("cosf"), _vec1("sinf")

T_F32, T_F16, T_BF16, T_PTQ1_0 = 0, 1, 30, 143


# ------------------------------------------------------------------ GGUF
def read_gguf(path: str):
    """GGUF v2/v3 (ref/bonsai-decoder/src/gguf.cpp): returns (metadata dict,
    {name: (type, ne list, bytes)}) over one read of the file."""
    buf = open(path, "rb").read()
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from("<" + fmt, buf, pos)
        pos += struct.calcsize("<" + fmt)
        return v[0]

    def string():
        nonlocal pos
        n = take("Q")
        s = buf[pos:pos + n].decode("utf-8")
        pos += n
        return s

    scalar = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}

    def value(t):
        if t == 8:
            return string()
        if t == 9:
            et, n = take("I"), take("Q")
            return [value(et) for _ in range(n)]
        return take(scalar[t])

    if buf[:4] != b"GGUF":
        raise ValueError("not a GGUF file")
    pos = 4
    version = take("I")
    if version not in (2, 3):
        raise ValueError(f"GGUF version {version}")
    n_tensors, n_kv = take("Q"), take("Q")
    kv = {}
    for _ in range(n_kv):
        k = string()
        kv[k] = value(take("I"))
    infos = []
    for _ in range(n_tensors):
        name = string()
        nd = take("I")
        ne = [take("Q") for _ in range(nd)]
        infos.append((name, ne, take("I"), take("Q")))
    align = int(kv.get("general.alignment", 32))
    data = (pos + align - 1) // align * align
    tensors = {}
    for name, ne, t, off in infos:
        n = int(np.prod(ne))
        nbytes = {T_F32: 4 * n, T_F16: 2 * n, T_BF16: 2 * n, T_PTQ1_0: n // 128 * 28}[t]
        tensors[name] = (t, ne, buf[data + off:data + off + nbytes])
    return kv, tensors


def _vec(t, raw):
    """F32 / F16 / BF16 tensor -> float32 (bd::to_f32, ref/bonsai-decoder/src/cpu_ops.cpp:139-146)."""
    if t == T_F32:
        return np.frombuffer(raw, dtype="<f4").copy()
    if t == T_F16:
        return np.frombuffer(raw, dtype="<f2").astype(np.float32)
    if t == T_BF16:
        return (np.frombuffer(raw, dtype="<u2").astype(np.uint32) << 16).view(np.float32)
    raise ValueError(f"vector tensor type {t}")


def _round_bf16(x):
    """bd::f32_to_bf16 then back (ref/bonsai-decoder/src/types.cpp:64-70)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    r = np.where(nan, ((u >> 16) | 0x40) << 16, r)
    return r.astype(np.uint32).view(np.float32)


def _seq_sum(a, axis=-1):
    """Sequential float32 sum along `axis` (the emulator's `s += ...` order)."""
    return np.cumsum(np.asarray(a, np.float32), axis=axis, dtype=np.float32).take(-1, axis=axis)


def _silu(x):
    x = np.asarray(x, np.float32)
    return (x / (np.float32(1) + expf(-x))).astype(np.float32)


def _sigmoid(x):
    x = np.asarray(x, np.float32)
    return (np.float32(1) / (np.float32(1) + expf(-x))).astype(np.float32)


def _softplus(x):
    x = np.float32(x)
    return x if x > 20.0 else log1pf(expf(x))


def _fwht(x, block):
    """bd::fwht per block (cpu_ops.cpp:76-88): butterflies in stage order, then * 1/sqrtf(block)."""
    y = np.array(x, np.float32).reshape(-1, block)
    length = 1
    while length < block:
        y = y.reshape(y.shape[0], -1, 2, length)
        a, b = y[:, :, 0, :].copy(), y[:, :, 1, :].copy()
        y[:, :, 0, :] = a + b
        y[:, :, 1, :] = a - b
        y = y.reshape(-1, block)
        length <<= 1
    return (y * (np.float32(1) / np.sqrt(np.float32(block)))).reshape(-1).astype(np.float32)


def _l2norm(x, eps):
    """bd::l2norm (cpu_ops.cpp:124-129)."""
    s = float(np.cumsum(np.asarray(x, np.float64) ** 2)[-1])
    scale = np.float32(1) / np.float32(max(np.float32(np.sqrt(np.float32(s))), np.float32(eps)))
    return (np.asarray(x, np.float32) * scale).astype(np.float32)


class Matrix:
    """A PTQ1_0 matrix as the reference's T2 codes / scales (btf::repack) plus its input transform."""

    def __init__(self, orc, raw, ne, hx):
        self.K, self.N = int(ne[0]), int(ne[1])
        src = np.frombuffer(raw, dtype=np.uint8).reshape(self.N, -1)
        self.codes, self.scales = orc.repack_t2(src, self.N, self.K)
        self.hx = hx  # (block, (perm_hd, perm_nk, perm_rep), signs) or None


class DecodeOracle:
    """Batch-1 decode steps of a qwen35 GGUF, restating the reference emulator."""

    def __init__(self, orc, path: str, n_ctx: int = 64, round_q_f16: bool = True):
        self.orc, self.n_ctx, self.round_q = orc, n_ctx, round_q_f16
        kv, ts = read_gguf(path)
        assert kv["general.architecture"] == "qwen35"
        p = "qwen35."
        g = lambda k, d=None: kv.get(p + k, d)
        self.L, self.E, self.F = g("block_count"), g("embedding_length"), g("feed_forward_length")
        self.L -= g("nextn_predict_layers", 0)  # MTP blocks are not run in the main pass
        self.H, self.HK = g("attention.head_count"), g("attention.head_count_kv")
        self.D = g("attention.key_length", self.E // self.H)
        self.R = g("rope.dimension_count", self.D)
        self.rope_base = np.float32(g("rope.freq_base", 10000.0))
        self.eps = np.float32(g("attention.layer_norm_rms_epsilon"))
        self.KC, self.DK, self.NK, self.NV = g("ssm.conv_kernel"), g("ssm.state_size"), g("ssm.group_count"), \
            g("ssm.time_step_rank")
        self.DI = g("ssm.inner_size")
        self.DV, self.QK = self.DI // self.NV, self.DK * self.NK
        self.C = 2 * self.QK + self.DI
        interval = g("full_attention_interval", 4)
        # prism Hadamard metadata (model.cpp:100-156)
        block, folded, signs, grouped, inverse = 0, set(), {}, False, False
        if kv.get("prism.hadamard.version", 0):
            block = kv["prism.hadamard.block_size"]
            folded = set(kv["prism.hadamard.weight_names"])
            if kv["prism.hadamard.sign_mode"] == "explicit":
                off, vals = 0, kv["prism.hadamard.sign_values"]
                for w in kv["prism.hadamard.sign_widths"]:
                    signs[w] = np.array(vals[off:off + w], np.float32)
                    off += w
            grouped = bool(kv.get("prism.hadamard.gdn_v_grouped", False))
            inverse = "token_embd.weight" in kv.get("prism.hadamard.inverse_weight_names", [])
            if kv.get("prism.hadamard.tied_output", False):
                folded.add("token_embd.weight")

        def hx(name, width):
            if name not in folded:
                return None
            perm = (0, 0, 0)
            if grouped and ".ssm_out." in name:
                perm = (width // self.NV, self.NK, self.NV // self.NK)
            return block, perm, signs.get(width)

        def mat(name):
            t, ne, raw = ts[name]
            return Matrix(orc, raw, ne, hx(name, int(ne[0])))

        def vec(name):
            t, ne, raw = ts[name]
            return _vec(t, raw)

        t, ne, raw = ts["token_embd.weight"]
        self.V = int(ne[1])
        self.embd = Matrix(orc, raw, ne, None)
        self.inv = (block, signs.get(self.E)) if inverse else None
        self.out_norm = vec("output_norm.weight")
        self.output = mat("output.weight" if "output.weight" in ts else "token_embd.weight")
        self.layers = []
        for il in range(self.L):
            b = f"blk.{il}."
            lay = dict(rec=((il + 1) % interval) != 0, attn_norm=vec(b + "attn_norm.weight"),
                       post_norm=vec(b + "post_attention_norm.weight"), gate=mat(b + "ffn_gate.weight"),
                       up=mat(b + "ffn_up.weight"), down=mat(b + "ffn_down.weight"))
            if lay["rec"]:
                lay.update(qkv=mat(b + "attn_qkv.weight"), zg=mat(b + "attn_gate.weight"),
                           alpha=vec(b + "ssm_alpha.weight").reshape(self.NV, self.E),
                           beta=vec(b + "ssm_beta.weight").reshape(self.NV, self.E),
                           ab_bf16=ts[b + "ssm_alpha.weight"][0] == T_BF16,
                           ssm_a=vec(b + "ssm_a"), ssm_dt=vec(b + "ssm_dt.bias"),
                           conv_w=vec(b + "ssm_conv1d.weight").reshape(self.C, self.KC),
                           ssm_norm=vec(b + "ssm_norm.weight"), out=mat(b + "ssm_out.weight"))
            else:
                lay.update(wq=mat(b + "attn_q.weight"), wk=mat(b + "attn_k.weight"), wv=mat(b + "attn_v.weight"),
                           wo=mat(b + "attn_output.weight"), q_norm=vec(b + "attn_q_norm.weight"),
                           k_norm=vec(b + "attn_k_norm.weight"))
            self.layers.append(lay)
        self.reset()

    def reset(self) -> None:
        self.pos = 0
        for lay in self.layers:
            if lay["rec"]:
                lay["conv"] = np.zeros((self.KC - 1, self.C), np.float32)
                lay["ssm"] = np.zeros((self.NV, self.DV, self.DK), np.float32)
            else:
                lay["kc"] = np.zeros((self.n_ctx, self.HK * self.D), np.float16)
                lay["vc"] = np.zeros((self.n_ctx, self.HK * self.D), np.float16)

    # ---- the emulator's prep (emu_decoder.cpp:121-140) and GEMV (:143-165)
    def _prep(self, x, normw, m: Matrix):
        block, perm, signs = m.hx if m.hx else (0, (0, 0, 0), None)
        q, d, s, xn = self.orc.prep_rows(np.asarray(x, np.float32)[None, :], normw, float(self.eps), block, perm, signs)
        return (q, d, s), xn[0]

    def _gemv(self, m: Matrix, a, y=None):
        q, d, s = a
        out = self.orc.gemv(m.codes, m.scales, m.K, q, d, s, y=None if y is None else y[None, :].copy(),
                            add=y is not None)
        return out[0]

    def step(self, token: int):
        """One token: (greedy next token, logits float32 [V])."""
        if self.pos >= self.n_ctx:
            raise RuntimeError("context full")
        E = self.E
        # embedding: decode the packed row, inverse transform (WHT then signs)
        if not 0 <= token < self.V:
            raise ValueError("token id out of range")
        codes = self._row_codes(self.embd, token).astype(np.float32)
        sc = self.embd.scales[token].view(np.float16).astype(np.float32)
        x = (codes * np.repeat(sc, 128)).astype(np.float32)
        if self.inv:
            block, signs = self.inv
            x = _fwht(x, block)
            if signs is not None:
                x = (x * signs).astype(np.float32)
        for lay in self.layers:
            if lay["rec"]:
                a, xn = self._prep(x, lay["attn_norm"], lay["qkv"])
                x = self._gdn(lay, a, xn, x)
            else:
                a, _ = self._prep(x, lay["attn_norm"], lay["wq"])
                x = self._attn(lay, a, x)
            a, _ = self._prep(x, lay["post_norm"], lay["gate"])
            gv = self._gemv(lay["gate"], a)
            uv = self._gemv(lay["up"], a)
            gv = (_silu(gv) * uv).astype(np.float32)
            a, _ = self._prep(gv, None, lay["down"])
            x = self._gemv(lay["down"], a, y=x)
        a, _ = self._prep(x, self.out_norm, self.output)
        logits = self._gemv(self.output, a)
        self.pos += 1
        return int(np.argmax(logits)), logits

    def _row_codes(self, m: Matrix, row: int):
        """Trits of one row of a T2 matrix (btf::packed_code - 1), through the C oracle."""
        cr = np.ascontiguousarray(m.codes[row])
        return np.array([self.orc.L.orc_t2_code(cr.ctypes.data, e) - 1 for e in range(m.K)], np.int32)

    def _gdn(self, lay, a, xn, x):
        C, DK, DV, NK, NV, QK = self.C, self.DK, self.DV, self.NK, self.NV, self.QK
        qkv = self._gemv(lay["qkv"], a)
        z = self._gemv(lay["zg"], a)
        xr = _round_bf16(xn) if lay["ab_bf16"] else xn
        sa = _seq_sum(lay["alpha"] * xr[None, :], axis=1)
        sb = _seq_sum(lay["beta"] * xr[None, :], axis=1)
        beta = _sigmoid(sb)
        g = np.array([_softplus(np.float32(sa[h] + lay["ssm_dt"][h])) * lay["ssm_a"][h] for h in range(NV)], np.float32)
        # conv (K taps) + silu, state shift (emu_decoder.cpp:251-264)
        st, w = lay["conv"], lay["conv_w"]
        s = np.zeros(C, np.float32)
        for i in range(self.KC - 1):
            s = (s + st[i] * w[:, i]).astype(np.float32)
        s = (s + qkv * w[:, self.KC - 1]).astype(np.float32)
        st[:-1] = st[1:].copy()
        st[-1] = qkv
        cv = _silu(s)
        # gated delta rule + gated RMSNorm per v-head (:266-298)
        o = np.zeros(self.DI, np.float32)
        qscale = np.float32(1) / np.sqrt(np.float32(DK))
        for h in range(NV):
            kh = h % NK
            q = _l2norm(cv[kh * DK:(kh + 1) * DK], self.eps)
            k = _l2norm(cv[QK + kh * DK:QK + (kh + 1) * DK], self.eps)
            v = cv[2 * QK + h * DV:2 * QK + (h + 1) * DV]
            col = lay["ssm"][h]  # [DV][DK]
            col *= expf(g[h])
            kv = _seq_sum(col * k[None, :], axis=1)
            dl = ((v - kv) * beta[h]).astype(np.float32)
            col += (k[None, :] * dl[:, None]).astype(np.float32)
            oh = (_seq_sum(col * q[None, :], axis=1) * qscale).astype(np.float32)
            oh = self.orc.rmsnorm(oh, lay["ssm_norm"], float(self.eps))
            o[h * DV:(h + 1) * DV] = (oh * _silu(z[h * DV:(h + 1) * DV])).astype(np.float32)
        b, _ = self._prep(o, None, lay["out"])
        return self._gemv(lay["out"], b, y=x)

    def _rope(self, hv, p):
        theta_scale = np.float32(_libm.powf(float(self.rope_base), float(np.float32(-2.0) / np.float32(self.R))))
        theta = np.float32(p)
        out = hv.copy()
        half = self.R // 2
        for ic in range(half):
            c, s = cosf(theta), sinf(theta)
            x0, x1 = hv[ic], hv[ic + half]
            out[ic] = x0 * c - x1 * s
            out[ic + half] = x0 * s + x1 * c
            theta = np.float32(theta * theta_scale)
        return out

    def _attn(self, lay, a, x):
        D, H, HK = self.D, self.H, self.HK
        kvw = HK * D
        qf = self._gemv(lay["wq"], a)
        k = self._gemv(lay["wk"], a)
        v = self._gemv(lay["wv"], a)
        p = self.pos
        q = np.zeros(H * D, np.float32)
        for h in range(H):
            qh = self._rope(self.orc.rmsnorm(qf[h * 2 * D:h * 2 * D + D], lay["q_norm"], float(self.eps)), p)
            if self.round_q:
                qh = qh.astype(np.float16).astype(np.float32)
            q[h * D:(h + 1) * D] = qh
        for h in range(HK):
            k[h * D:(h + 1) * D] = self._rope(self.orc.rmsnorm(k[h * D:(h + 1) * D], lay["k_norm"], float(self.eps)), p)
        lay["kc"][p] = k.astype(np.float16)
        lay["vc"][p] = v.astype(np.float16)
        T = p + 1
        scale = np.float32(1) / np.sqrt(np.float32(D))
        grp = H // HK
        o = np.zeros(H * D, np.float32)
        for h in range(H):
            gk = h // grp
            kt = lay["kc"][:T, gk * D:(gk + 1) * D].astype(np.float32)
            vt = lay["vc"][:T, gk * D:(gk + 1) * D].astype(np.float32)
            sc = (_seq_sum(q[h * D:(h + 1) * D][None, :] * kt, axis=1) * scale).astype(np.float32)
            mx = np.max(sc)
            e = expf(sc - mx)
            tot = _seq_sum(e)
            oh = np.cumsum(e[:, None] * vt, axis=0, dtype=np.float32)[-1]
            gate = qf[h * 2 * D + D:h * 2 * D + 2 * D]
            o[h * D:(h + 1) * D] = (oh / tot * _sigmoid(gate)).astype(np.float32)
        b, _ = self._prep(o, None, lay["wo"])
        return self._gemv(lay["wo"], b, y=x)
