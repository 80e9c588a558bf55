"""CPU oracle of the whole decoder (TEST INFRASTRUCTURE ONLY).

Restates the TFJS reference block and engine (browser-tfjs-webgl-distribution/runtime/
official-w4a16-layer0.js:129-373, tfjs-reference-engine.js:246-396) with the WGSL
runtime's formulas where they differ (custom-webgpu/gpu-runtime.js: GELU clamp :1154,
RoPE angle :1197-1198, PLE mix :1259-1262, head softcap :1275), for one sequence.

It mirrors the rounding points of the bf16 activations the B200 path uses (inputs of
every W4A16 linear, q, K, V and the attention output are bf16) so greedy decoding can
be compared token for token.  Linear weights are the exact dequantised values
q * scale (official-w4a16.js:95, the reference's own f32 weights) for calls of at most
`gemm_rows` rows and their bf16 materialisation (roundFloat32ToBF16 of q * scale) above.
`gemm_rows=EXACT` (no limit) is the reference's arithmetic everywhere: the primary
comparison.  The default of 16 mirrors where the GPU switches from the decode GEMV
(exact q * scale) to the tcgen05 GEMM (bf16 weights): a secondary, tighter check of the
GEMM path.  Matmuls run in float32/float64 BLAS, reductions in f32/f64.  One instance
holds one sequence at a time; `state()` / `set_state()` swap sequences in and out while
the dequantised weights stay shared.
"""
from __future__ import annotations

import math

import numpy as np

from . import bf16_bits_to_f32, f32_to_bf16_bits
from . import numpy_oracle as npo


EXACT = 1 << 62  # gemm_rows that keeps the exact f32 weights for every call


def bf16r(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, np.float32)))


def rms(x: np.ndarray, scale: np.ndarray | None, eps: float) -> np.ndarray:
    """RMS_SHADER (gpu-runtime.js:1104-1118), rmsnorm.js:34-45."""
    x = np.asarray(x, np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    y = x * (np.float32(1.0) / np.sqrt(ms + np.float32(eps)))
    return y * scale if scale is not None else y


def gelu(x: np.ndarray) -> np.ndarray:
    """geluTanh (official-w4a16-layer0.js:6-14) with the ±10 clamp of GELU_MUL (:1154)."""
    x = np.asarray(x, np.float32)
    z = np.float32(0.7978845608028654) * (x + np.float32(0.044715) * x * x * x)
    return np.float32(0.5) * x * (np.float32(1.0) + np.tanh(np.clip(z, -10, 10)))


def norm_rope(x: np.ndarray, scale: np.ndarray, pos: np.ndarray, rope_angles: int, base: float, eps: float):
    """NORM_ROPE_SHADER (gpu-runtime.js:1175-1202) = RMSNorm + applyRoPE (rope.js:10-68)."""
    hd = x.shape[-1]
    half = hd // 2
    y = rms(x, scale, eps)
    a, b = y[..., :half], y[..., half:]
    i = np.arange(half, dtype=np.float32)
    theta = pos.astype(np.float32)[:, None] / np.power(np.float32(base), np.float32(2.0) * i / np.float32(hd))
    theta = theta.astype(np.float32)
    sn = np.where(i < rope_angles, np.sin(theta), 0).astype(np.float32)
    cs = np.where(i < rope_angles, np.cos(theta), 1).astype(np.float32)
    if y.ndim == 3:
        sn, cs = sn[:, None, :], cs[:, None, :]
    return np.concatenate([a * cs - b * sn, b * cs + a * sn], axis=-1).astype(np.float32)


class OracleModel:
    """Greedy decoder of one sequence with a KV cache, mirroring Gemma4Model."""

    def __init__(self, cfg, w: dict, max_seq: int = 512, gemm_rows: int = 16):
        self.cfg, self.max_seq, self.gemm_rows = cfg, max_seq, gemm_rows
        self.layers = []
        for i, lw in enumerate(w["layers"]):
            s = cfg.spec(i)
            L = {"spec": s, "skip": np.float32(lw["skip"])}
            for name in ("qkv", "o", "gu", "down", "pg", "pp"):
                L[name] = self._lin(*lw[name])
            for n in ("n_in", "n_pa", "n_pf", "n_pff", "n_pple", "qn", "kn"):
                L[n] = np.asarray(lw[n], np.float32)
            self.layers.append(L)
        self.top = self._lin(*w["top"])
        self.ple_norm = np.asarray(w["ple_norm"], np.float32)
        self.final_norm = np.asarray(w["final_norm"], np.float32)
        self.embed_bits = w["embed"]
        self.ple_packed, self.ple_scales = w["ple_packed"], w["ple_scales"]
        self.reset()

    @staticmethod
    def _lin(packed, scales):
        return {"packed": np.asarray(packed), "scales": np.asarray(scales)}

    @staticmethod
    def _weights(lin, key):
        """Dequantised weights, built on first use (exact q*s, or its bf16 rounding)."""
        if "exact" not in lin:
            lin["exact"] = npo.dequant_w4a16(lin["packed"], lin["scales"])
        if key == "bf16" and "bf16" not in lin:
            lin["bf16"] = bf16r(lin["exact"])
        return lin[key]

    def fresh_state(self) -> dict:
        """An empty sequence: position 0 and zeroed K/V caches of every non-shared layer."""
        st = {"pos": 0, "k": {}, "v": {}}
        for i, L in enumerate(self.layers):
            if not L["spec"]["shared"]:
                hd = L["spec"]["hd"]
                st["k"][i] = np.zeros((self.max_seq, hd), np.float32)
                st["v"][i] = np.zeros((self.max_seq, hd), np.float32)
        return st

    def state(self) -> dict:
        """The current sequence (position and K/V caches), to swap sequences in and out
        while the dequantised weights stay shared."""
        return {"pos": self.pos, "k": self.k, "v": self.v}

    def set_state(self, st: dict) -> None:
        self.pos, self.k, self.v = st["pos"], st["k"], st["v"]

    def reset(self):
        self.set_state(self.fresh_state())

    def linear(self, lin, x):
        w = self._weights(lin, "bf16" if x.shape[0] > self.gemm_rows else "exact")
        return (bf16r(x) @ w.T).astype(np.float32)

    def attention(self, q, kc, vc, pos, keylen, full):
        """scaledDotProductAttention (official-w4a16-layer0.js:30-62), scale 1.0, mask of
        QK_SHADER (gpu-runtime.js:1214-1217)."""
        cfg = self.cfg
        kk = kc[:keylen].astype(np.float64)
        vv = vc[:keylen].astype(np.float64)
        R, Hh, D = q.shape
        logits = (q.astype(np.float64).reshape(R * Hh, D) @ kk.T).reshape(R, Hh, keylen)
        key = np.arange(keylen)[None, :]
        qp = pos[:, None]
        valid = key <= qp
        if not full:
            valid &= (key + cfg.window) > qp
        logits = np.where(valid[:, None, :], logits, -np.inf)
        logits -= logits.max(-1, keepdims=True)
        p = np.exp(logits)
        p /= p.sum(-1, keepdims=True)
        return bf16r((p.reshape(R * Hh, keylen) @ vv).reshape(R, Hh, D).astype(np.float32))

    def forward(self, ids) -> tuple[int, np.ndarray]:
        """Appends ids at the current position; returns (greedy next id, capped logits of the last row)."""
        cfg = self.cfg
        ids = np.asarray(ids, np.int64)
        T = ids.size
        H, P, Lc = cfg.hidden, cfg.ple_dim, cfg.layers
        pos = self.pos + np.arange(T)
        # inputBuffers / scale / w4(topProj) / scale / pleMix (gemma4-webgpu.js:316-321)
        h = bf16_bits_to_f32(self.embed_bits[ids]) * np.float32(math.sqrt(H))
        tok = npo.ple_read_rows(self.ple_packed, self.ple_scales, ids)
        proj = self.linear(self.top, h) * np.float32(1.0 / math.sqrt(H))
        proj = proj.reshape(T, Lc, P)
        per_layer = ((rms(proj, self.ple_norm, cfg.eps) + tok.reshape(T, Lc, P) * np.float32(math.sqrt(P)))
                     * np.float32(0.7071067811865476)).astype(np.float32)
        for i, L in enumerate(self.layers):
            s = L["spec"]
            hd = s["hd"]
            x = rms(h, L["n_in"], cfg.eps)
            qkv = self.linear(L["qkv"], x)
            q = qkv[:, :cfg.heads * hd].reshape(T, cfg.heads, hd)
            q = bf16r(norm_rope(q, L["qn"], pos, s["rope_angles"], s["rope_base"], cfg.eps))
            src = s["kv_src"] if s["shared"] else i
            if not s["shared"]:
                k = qkv[:, cfg.heads * hd:(cfg.heads + 1) * hd]
                v = qkv[:, (cfg.heads + 1) * hd:(cfg.heads + 2) * hd]
                self.k[i][pos] = bf16r(norm_rope(k, L["kn"], pos, s["rope_angles"], s["rope_base"], cfg.eps))
                self.v[i][pos] = bf16r(rms(v, None, cfg.eps))
            attn = self.attention(q, self.k[src], self.v[src], pos, self.pos + T, s["full"])
            o = self.linear(L["o"], attn.reshape(T, -1))
            h = (h + rms(o, L["n_pa"], cfg.eps)).astype(np.float32)
            gu = self.linear(L["gu"], rms(h, L["n_pf"], cfg.eps))
            inter = s["inter"]
            act = gelu(gu[:, :inter]) * gu[:, inter:]
            d = self.linear(L["down"], act)
            h = (h + rms(d, L["n_pff"], cfg.eps)).astype(np.float32)
            pg = self.linear(L["pg"], h)
            pa = gelu(pg) * per_layer[:, i, :]
            pp = self.linear(L["pp"], pa)
            h = ((h + rms(pp, L["n_pple"], cfg.eps)) * L["skip"]).astype(np.float32)
        self.pos += T
        # final norm, tied bf16 head with softcap, greedy (gemma4-webgpu.js:404-478)
        xf = bf16r(rms(h[-1:], self.final_norm, cfg.eps))
        if not hasattr(self, "_emb"):
            self._emb = bf16_bits_to_f32(self.embed_bits)
        raw = (xf @ self._emb.T)[0].astype(np.float32)
        capped = (np.tanh(raw / np.float32(cfg.softcap)) * np.float32(cfg.softcap)).astype(np.float32)
        return int(np.argmax(capped)), capped
