"""Gemma 4 E2B-shaped text decoder driven through the g4w4 C ABI.

This is the caller side of the drop-in boundary: a Python mirror of the reference's
model graph (`Gemma4WebGPU`, custom-webgpu/gemma4-webgpu.js) that issues the same
operators in the same order (encodeLayer :215-310, forward :311-412, logits :413-440,
greedy :441-480), with the reference's fusions of adjacent row-wise ops and two
structural changes for B200:

  * q, k and v (and gate and up) of a layer are one W4A16 linear each, their weight
    rows concatenated at load time (the same bits, one launch);
  * positions live on the device (`seq_pos`), K/V are appended by the q/k/v
    post-processing kernel, and the next token is picked on the device, so a whole
    decode step is one CUDA graph with no host round trip.

A batch of independent sequences decodes together: row b of a decode step is
sequence b.  `ModelConfig()` is the benchmark configuration (35 layers, hidden 1536,
MLP 6144, 8 q heads / 1 KV head, head_dim 256, window 512 on 4 of 5 layers, PLE 256
per layer, vocab 262144, tied bf16 head); `ModelConfig.reference_spec()` is the
checkpoint's own spec (head_dim 512 and rope 1e6 / 0.25 on global layers, MLP 12288
from layer 15, layers 15-34 reuse the KV of layers 13 / 14; gemma4-webgpu.js:65-77).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, replace

import numpy as np
import torch

from . import _lib
from ._lib import G4Planes, G4Rows, call
from .runtime import Context, G4Error, KVCache, PleW4Table, W4Linear


@dataclass(frozen=True)
class ModelConfig:
    hidden: int = 1536
    layers: int = 35
    heads: int = 8
    vocab: int = 262144
    ple_dim: int = 256
    window: int = 512
    head_dim: int = 256
    head_dim_global: int = 256
    intermediate: int = 6144
    intermediate_late: int = 6144      # layers >= first_shared (12288 in the checkpoint)
    kv_share: bool = False             # layers >= first_shared reuse the KV of the last local/global layer
    first_shared: int = 15
    rope_local: float = 10000.0
    rope_global: float = 1000000.0
    rope_prop_global: float = 0.25
    eps: float = 1e-6
    softcap: float = 30.0

    @staticmethod
    def reference_spec() -> "ModelConfig":
        return ModelConfig(head_dim_global=512, intermediate_late=12288, kv_share=True)

    def small(self, **kw) -> "ModelConfig":
        return replace(self, **kw)

    def spec(self, i: int) -> dict:
        """gemma4-webgpu.js:65-77."""
        full = (i + 1) % 5 == 0
        hd = self.head_dim_global if full else self.head_dim
        shared = self.kv_share and i >= self.first_shared
        src = None
        if shared:  # the last non-shared layer of the same attention type (13 / 14 in the checkpoint)
            src = max(j for j in range(self.first_shared) if ((j + 1) % 5 == 0) == full)
        return {
            "full": full, "hd": hd,
            "inter": self.intermediate_late if i >= self.first_shared else self.intermediate,
            "shared": shared, "kv_src": src,
            "rope_base": self.rope_global if full else self.rope_local,
            "rope_angles": int(math.floor((self.rope_prop_global if full else 1.0) * hd / 2)),
        }


# ----------------------------------------------------------------- weights ---
def _w4(rng, n, k, sigma, symmetric=True):
    """Packed int32 [n, k/8] + bf16 scales [n, k/32].  symmetric: q uniform in [-7, 7]
    (nibbles 1..15, zero mean); otherwise uniform over all 16 nibbles ([-8, 7])."""
    if symmetric:
        nib = rng.integers(1, 16, size=(n, k), dtype=np.uint8).astype(np.uint32)
        words = np.zeros((n, k // 8), np.uint32)
        for j in range(8):
            words |= nib[:, j::8] << np.uint32(4 * j)
        packed = words.view(np.int32)
    else:
        packed = rng.integers(0, 2**32, size=(n, k // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    s = np.abs(rng.standard_normal((n, k // 32), dtype=np.float32)) * np.float32(sigma)
    return packed, _bf16_bits(s)


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _norm(rng, n, center=1.0, spread=0.1):
    return (center * (1.0 + spread * rng.standard_normal(n))).astype(np.float32)


def random_weights(cfg: ModelConfig, seed: int = 0, sigma: float = 0.02, embed_sigma: float = 0.05,
                   qk_norm: float = 0.3, embed_tail: float = 0.0, post_norm: float = 1.0,
                   ple_post_norm: float | None = None, skip: tuple[float, float] = (0.5, 1.0)) -> dict:
    """Seeded random weights of the architecture on the host (numpy), in the
    checkpoint's formats: W4 linears as compressed-tensors packed int32 + bf16 scales,
    the tied embedding bf16, the PLE table as the W4 shard format, norms f32."""
    rng = np.random.default_rng(seed)
    H, L, P = cfg.hidden, cfg.layers, cfg.ple_dim
    w = {"layers": []}
    for i in range(L):
        s = cfg.spec(i)
        hd, inter = s["hd"], s["inter"]
        lw = {}
        qn = cfg.heads * hd + (0 if s["shared"] else 2 * hd)
        lw["qkv"] = _w4(rng, qn, H, sigma)
        lw["o"] = _w4(rng, H, cfg.heads * hd, sigma)
        lw["gu"] = _w4(rng, 2 * inter, H, sigma)
        lw["down"] = _w4(rng, H, inter, sigma)
        lw["pg"] = _w4(rng, P, H, sigma)
        lw["pp"] = _w4(rng, H, P, sigma)
        for n in ("n_in", "n_pf"):
            lw[n] = _norm(rng, H)
        for n in ("n_pa", "n_pff", "n_pple"):   # scale of each residual update
            lw[n] = _norm(rng, H, post_norm if n != "n_pple" or ple_post_norm is None else ple_post_norm)
        lw["qn"] = _norm(rng, hd, qk_norm)
        lw["kn"] = _norm(rng, hd, qk_norm)
        lw["skip"] = float(rng.uniform(*skip))
        w["layers"].append(lw)
    w["top"] = _w4(rng, L * P, H, sigma)
    w["ple_norm"] = _norm(rng, P)
    w["final_norm"] = _norm(rng, H)
    emb = rng.standard_normal((cfg.vocab, H), dtype=np.float32) * np.float32(embed_sigma)
    if embed_tail:  # log-normal row norms: the largest logits stand apart (clear greedy margins)
        emb *= np.exp(np.float32(embed_tail) * rng.standard_normal((cfg.vocab, 1), dtype=np.float32))
    w["embed"] = _bf16_bits(emb)
    del emb
    # PLE: two's complement nibbles in [-7, 7], bf16 scales |N(0, 0.05)| (benchmark config 2)
    q = rng.integers(-7, 8, size=(cfg.vocab, L * P), dtype=np.int8)
    nib = (q & 0xF).astype(np.uint8)
    w["ple_packed"] = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    w["ple_scales"] = _bf16_bits(np.abs(rng.standard_normal((cfg.vocab, L * P // 32), dtype=np.float32)) * 0.05)
    return w


def random_weights_device(cfg: ModelConfig, seed: int = 0, sigma: float = 0.02, embed_sigma: float = 0.05,
                          qk_norm: float = 0.3, device="cuda") -> dict:
    """Same architecture and distributions, generated on the GPU (for benchmarks)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, L, P = cfg.hidden, cfg.layers, cfg.ple_dim

    def w4(n, k):
        packed = torch.randint(-2**31, 2**31 - 1, (n, k // 8), device=device, dtype=torch.int32, generator=g)
        sc = torch.randn((n, k // 32), device=device, generator=g).abs_().mul_(sigma).to(torch.bfloat16)
        return packed, sc

    def norm(n, center=1.0):
        return (center * (1.0 + 0.1 * torch.randn(n, device=device, generator=g))).float()

    w = {"layers": []}
    for i in range(L):
        s = cfg.spec(i)
        hd, inter = s["hd"], s["inter"]
        lw = {"qkv": w4(cfg.heads * hd + (0 if s["shared"] else 2 * hd), H), "o": w4(H, cfg.heads * hd),
              "gu": w4(2 * inter, H), "down": w4(H, inter), "pg": w4(P, H), "pp": w4(H, P)}
        for n in ("n_in", "n_pa", "n_pf", "n_pff", "n_pple"):
            lw[n] = norm(H)
        lw["qn"], lw["kn"] = norm(hd, qk_norm), norm(hd, qk_norm)
        lw["skip"] = float(0.5 + 0.5 * torch.rand(1, generator=g, device=device).item())
        w["layers"].append(lw)
    w["top"] = w4(L * P, H)
    w["ple_norm"], w["final_norm"] = norm(P), norm(H)
    w["embed"] = (torch.randn((cfg.vocab, H), device=device, generator=g) * embed_sigma).to(torch.bfloat16)
    q = torch.randint(-7, 8, (cfg.vocab, L * P // 2, 2), device=device, dtype=torch.int16, generator=g)
    nib = (q & 0xF).to(torch.uint8)
    w["ple_packed"] = (nib[..., 0] | (nib[..., 1] << 4)).contiguous()
    del q, nib
    w["ple_scales"] = torch.randn((cfg.vocab, L * P // 32), device=device, generator=g).abs_().mul_(0.05).to(torch.bfloat16)
    return w


def interleave_geglu(a, inter: int):
    """Rows [gate (inter); up (inter)] -> slabs of 64 gate rows then the 64 matching up rows
    (the layout g4_linear_w4a16_geglu reads); numpy or torch."""
    g, u = a[:inter], a[inter:]
    rest = tuple(a.shape[1:])
    if isinstance(a, torch.Tensor):
        return torch.stack([g.reshape(inter // 64, 64, *rest), u.reshape(inter // 64, 64, *rest)], dim=1).reshape(
            2 * inter, *rest).contiguous()
    return np.ascontiguousarray(np.stack([g.reshape(inter // 64, 64, *rest), u.reshape(inter // 64, 64, *rest)],
                                         axis=1).reshape(2 * inter, *rest))


def _dev_f32(a, device):
    return (a if isinstance(a, torch.Tensor) else torch.from_numpy(np.asarray(a))).to(device=device, dtype=torch.float32).contiguous()


def _ptr(t):
    return C.c_void_p(t.data_ptr())


class Dense:
    """g4_dense: the tied bf16 embedding / LM head."""

    def __init__(self, ctx: Context, w):
        self.ctx = ctx
        N, K = int(w.shape[0]), int(w.shape[1])
        if isinstance(w, torch.Tensor):
            w = w.contiguous()
            src, on_dev = C.c_void_p(w.data_ptr()), int(w.is_cuda)
        else:
            w = np.ascontiguousarray(w)
            src, on_dev = C.c_void_p(w.ctypes.data), 0
        h = C.c_void_p()
        call("g4_dense_create", ctx.handle, src, K, N, on_dev, C.byref(h))
        self.handle, self.K, self.N = h, K, N
        p = C.c_void_p()
        call("g4_dense_weights", h, C.byref(p))
        self.weights_ptr = p

    def close(self):
        if getattr(self, "handle", None):
            _lib.load().g4_dense_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Decoder:
    """g4_decoder: the whole batch-1 decode step of a Gemma4Model as one persistent launch
    (one CTA per SM, phases separated by grid barriers, weights streamed ahead of each
    barrier).  Built from the model's own device objects; see include/g4w4.h."""

    def __init__(self, m: "Gemma4Model"):
        cfg = m.cfg
        n = len(m.layers)
        self._keep = []
        layers = (_lib.G4DecoderLayer * n)()
        for i, L in enumerate(m.layers):
            s = L["spec"]
            nxt = m.layers[i]["n_in"]
            layers[i] = _lib.G4DecoderLayer(
                L["qkv"].handle, L["o"].handle, L["gu"].handle, L["down"].handle, L["pg"].handle, L["pp"].handle,
                nxt.data_ptr(), L["n_pa"].data_ptr(), L["n_pf"].data_ptr(), L["n_pff"].data_ptr(),
                L["n_pple"].data_ptr(), L["qn"].data_ptr(), L["kn"].data_ptr(), C.c_float(L["skip"]),
                L["kv"].handle, 0 if s["shared"] else 1, 1 if s["full"] else 0, s["rope_angles"],
                C.c_float(s["rope_base"]), s["inter"])
        desc = _lib.G4DecoderDesc(n, cfg.hidden, cfg.heads, cfg.ple_dim, cfg.window, cfg.vocab, C.c_float(cfg.eps),
                                  C.c_float(cfg.softcap), m.top.handle, m.ple_norm.data_ptr(),
                                  m.final_norm.data_ptr(), m.head.handle, m.ple.handle)
        h = C.c_void_p()
        call("g4_decoder_create", m.ctx.handle, C.byref(desc), layers, C.byref(h))
        self.handle = h

    def step(self, ctx: Context, ids, seq_pos, nxt, val):
        call("g4_decoder_step", ctx.handle, self.handle, _ptr(ids), _ptr(seq_pos), _ptr(nxt), _ptr(val))

    def reset(self):
        call("g4_decoder_reset", self.handle)

    def close(self):
        if getattr(self, "handle", None):
            _lib.load().g4_decoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Gemma4Model:
    """Mirror of Gemma4WebGPU over libg4w4 (see the module docstring).

    persistent: decode steps of a single-sequence model (max_batch 1) run as one
    persistent g4_decoder launch instead of the ~430 operator launches of the op path
    (prefill and batched decode always use the operators).  Off by default: on B200 the
    operator chain with programmatic dependent launch measures faster (1.6 vs 3.0 ms per
    token at config 4), the persistent step paying ~10 us per grid-barrier phase.

    ring_kv: the caches of sliding-window layers keep each sequence's last window +
    max_rows - 1 positions (g4_kv_create_ring; the Node reference trims its sliding caches
    to the window, node-reference/src/attention.js:299-305) whenever that is smaller than
    max_seq; global layers keep every position."""

    def __init__(self, ctx: Context, cfg: ModelConfig, w: dict, max_batch: int = 1, max_seq: int = 512,
                 max_rows: int | None = None, pdl: bool = True, persistent: bool = False, ring_kv: bool = True):
        self.ctx, self.cfg = ctx, cfg
        self.persistent = persistent and max_batch == 1
        self._dec = None
        if pdl:  # the decode step is a long chain of this library's kernels on one stream
            ctx.set_pdl(True)
        self.max_batch, self.max_seq = max_batch, max_seq
        self.max_rows = max(max_rows or 0, max_batch, 1)
        dev = ctx.torch_device
        self.dev = dev
        # gemma4-webgpu.js:150-191 load(): linears, norms, caches, LM head
        self.layers = []
        for i, lw in enumerate(w["layers"]):
            s = cfg.spec(i)
            L = {"spec": s, "skip": float(lw["skip"])}
            for name in ("qkv", "o", "down", "pg", "pp"):
                L[name] = W4Linear(ctx, lw[name][0], lw[name][1], name=f"layers.{i}.{name}")
            # gate and up rows interleaved in 64-row blocks: GeGLU is fused into the linear
            L["gu"] = W4Linear(ctx, interleave_geglu(lw["gu"][0], s["inter"]), interleave_geglu(lw["gu"][1], s["inter"]),
                               name=f"layers.{i}.gu")
            for n in ("n_in", "n_pa", "n_pf", "n_pff", "n_pple", "qn", "kn"):
                L[n] = _dev_f32(lw[n], dev)
            L["kv"] = None if s["shared"] else self._cache(s, ring_kv)
            self.layers.append(L)
        for L in self.layers:
            if L["spec"]["shared"]:
                src = self.layers[L["spec"]["kv_src"]]
                assert src["spec"]["full"] == L["spec"]["full"], "a KV-shared layer reads a cache of its own kind"
                L["kv"] = src["kv"]
        self.top = W4Linear(ctx, w["top"][0], w["top"][1], name="per_layer_model_projection")
        self.ple_norm = _dev_f32(w["ple_norm"], dev)
        self.final_norm = _dev_f32(w["final_norm"], dev)
        self.head = Dense(ctx, w["embed"])
        self.ple = PleW4Table(ctx, w["ple_packed"], w["ple_scales"])
        self.seq_pos = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self._alloc(self.max_rows)
        self.graph = None
        self._capturing = False

    def _cache(self, spec: dict, ring_kv: bool) -> KVCache:
        """A layer's cache: a ring of window + max_rows - 1 slots per sequence for a sliding
        layer when that saves memory (a prefill of up to max_rows tokens then still finds
        every key its rows' windows need), else max_seq rows per sequence."""
        hd = spec["hd"]
        ring = max(self.cfg.window + self.max_rows - 1, 16384 // hd)
        if ring_kv and not spec["full"] and ring + 16384 // hd < self.max_seq:
            return KVCache(self.ctx, hd, self.max_seq, ring=ring, nseq=self.max_batch)
        return KVCache(self.ctx, hd, self.max_batch * self.max_seq)

    def kv_stride(self, kv: KVCache) -> int:
        """Rows per sequence of a layer cache (g4_attention_rows seq_stride)."""
        return kv.seq_rows if kv.ring else self.max_seq

    # ------------------------------------------------------------ buffers ---
    def _alloc(self, R):
        cfg, dev = self.cfg, self.dev
        hdm = max(cfg.head_dim, cfg.head_dim_global)
        im = max(cfg.intermediate, cfg.intermediate_late)
        LP = cfg.layers * cfg.ple_dim
        f32, b16 = torch.float32, torch.bfloat16
        self.buf = {
            "h": torch.empty((R, cfg.hidden), dtype=f32, device=dev),
            "x": torch.empty((R, cfg.hidden), dtype=b16, device=dev),
            "qkv": torch.empty((R, (cfg.heads + 2) * hdm), dtype=f32, device=dev),
            "q": torch.empty((R, cfg.heads * hdm), dtype=b16, device=dev),
            "attn": torch.empty((R, cfg.heads * hdm), dtype=b16, device=dev),
            "y": torch.empty((R, cfg.hidden), dtype=f32, device=dev),
            "gu": torch.empty((R, 2 * im), dtype=f32, device=dev),
            "act": torch.empty((R, im), dtype=b16, device=dev),
            "pg": torch.empty((R, cfg.ple_dim), dtype=f32, device=dev),
            "pa": torch.empty((R, cfg.ple_dim), dtype=b16, device=dev),
            "proj": torch.empty((R, LP), dtype=f32, device=dev),
            "tokple": torch.empty((R, LP), dtype=f32, device=dev),
            "per_layer": torch.empty((R, LP), dtype=f32, device=dev),
            "logits": torch.empty((self.max_batch, cfg.vocab), dtype=f32, device=dev),
            "ids": torch.zeros(R, dtype=torch.int32, device=dev),
            "next": torch.zeros(self.max_batch, dtype=torch.int32, device=dev),
            "val": torch.zeros(self.max_batch, dtype=f32, device=dev),
        }

    def reset(self):
        """resetCache (gemma4-webgpu.js:193-196)."""
        self.seq_pos.zero_()

    # ------------------------------------------------------------ forward ---
    def _w4(self, lin, x, rows, y):
        call("g4_linear_w4a16", self.ctx.handle, lin.handle, _ptr(x), rows, _ptr(y), 0)

    def _w4p(self, lin, x, rows) -> G4Planes:
        """The linear's f32 output left as split-K planes in the context workspace, read
        (and summed) by the row-wise operator that follows."""
        pl = G4Planes()
        call("g4_linear_w4a16_planes", self.ctx.handle, lin.handle, _ptr(x), rows, C.byref(pl))
        return pl

    def _forward(self, ids, rows, rmap: G4Rows, head_rows: int, head_x_row0: int):
        """Issues one forward of `rows` rows (ids: int32 device [rows]) and the greedy pick
        of `head_rows` rows starting at row head_x_row0 into buf["next"]."""
        cfg, b, h = self.cfg, self.buf, self.ctx.handle
        H, P, L = cfg.hidden, cfg.ple_dim, cfg.layers
        # inputBuffers + top-level embedding and PLE projection (gemma4-webgpu.js:198-213, :316-323)
        call("g4_embed", h, self.head.weights_ptr, cfg.vocab, H, _ptr(ids), rows, C.c_float(math.sqrt(H)),
             _ptr(b["h"]), _ptr(b["x"]))
        call("g4_ple_gather", h, self.ple.handle, _ptr(ids), rows, 1, _ptr(b["tokple"]), 0)
        self._w4(self.top, b["x"], rows, b["proj"])
        call("g4_ple_mix", h, _ptr(b["proj"]), C.c_float(1.0 / math.sqrt(H)), _ptr(self.ple_norm), _ptr(b["tokple"]),
             rows, L, P, C.c_float(cfg.eps), _ptr(b["per_layer"]))
        call("g4_rms", h, _ptr(b["h"]), _ptr(self.layers[0]["n_in"]), rows, H, C.c_float(cfg.eps), _ptr(b["x"]), 1)
        for i, Ly in enumerate(self.layers):
            s = Ly["spec"]
            hd = s["hd"]
            # encodeLayer (gemma4-webgpu.js:215-310)
            kv = Ly["kv"]
            kp, vp = C.c_void_p(), C.c_void_p()
            call("g4_kv_buffers", kv.handle, C.byref(kp), C.byref(vp))
            qkv = self._w4p(Ly["qkv"], b["x"], rows)
            if kv.ring and not s["shared"]:
                call("g4_qkv_post_kv", h, C.byref(qkv), cfg.heads, hd, _ptr(Ly["qn"]), _ptr(Ly["kn"]),
                     C.c_float(cfg.eps), s["rope_angles"], C.c_float(s["rope_base"]), C.byref(rmap), rows,
                     _ptr(b["q"]), kv.handle)
            else:
                call("g4_qkv_post_planes", h, C.byref(qkv), cfg.heads, hd, 0 if s["shared"] else 1,
                     _ptr(Ly["qn"]), _ptr(Ly["kn"]), C.c_float(cfg.eps), s["rope_angles"], C.c_float(s["rope_base"]),
                     C.byref(rmap), rows, _ptr(b["q"]), kp, vp, self.max_seq)
            call("g4_attention_rows", h, _ptr(b["q"]), kv.handle, rows, cfg.heads, hd, C.byref(rmap), self.kv_stride(kv),
                 0 if s["full"] else 1, cfg.window, _ptr(b["attn"]))
            y = self._w4p(Ly["o"], b["attn"], rows)
            call("g4_post_norm_add_planes", h, _ptr(b["h"]), C.byref(y), _ptr(Ly["n_pa"]), C.c_float(1.0),
                 _ptr(Ly["n_pf"]), rows, H, C.c_float(cfg.eps), _ptr(b["x"]))
            call("g4_linear_w4a16_geglu", h, Ly["gu"].handle, _ptr(b["x"]), rows, _ptr(b["act"]))
            y = self._w4p(Ly["down"], b["act"], rows)
            call("g4_post_norm_add_planes", h, _ptr(b["h"]), C.byref(y), _ptr(Ly["n_pff"]), C.c_float(1.0), None,
                 rows, H, C.c_float(cfg.eps), _ptr(b["x"]))
            # PLE gate + GELU x per-layer input (gemma4-webgpu.js:299-300); one launch up to 16 rows
            call("g4_linear_w4a16_gelu_ple", h, Ly["pg"].handle, _ptr(b["x"]), rows, _ptr(b["per_layer"]), i, L,
                 _ptr(b["pa"]))
            y = self._w4p(Ly["pp"], b["pa"], rows)
            w_next = self.layers[i + 1]["n_in"] if i + 1 < L else self.final_norm  # :404 final rms fused here
            call("g4_post_norm_add_planes", h, _ptr(b["h"]), C.byref(y), _ptr(Ly["n_pple"]), C.c_float(Ly["skip"]),
                 _ptr(w_next), rows, H, C.c_float(cfg.eps), _ptr(b["x"]))
        # logits + greedy (gemma4-webgpu.js:413-480)
        xh = b["x"][head_x_row0:head_x_row0 + head_rows]
        if head_rows > 16:  # batched: logits tiles reduced in the head kernel's epilogue, never stored
            call("g4_dense_argmax", h, self.head.handle, _ptr(xh), head_rows, C.c_float(cfg.softcap), _ptr(b["next"]),
                 _ptr(b["val"]))
        else:
            call("g4_dense_matmul", h, self.head.handle, _ptr(xh), head_rows, _ptr(b["logits"]))
            call("g4_softcap_argmax", h, _ptr(b["logits"]), head_rows, cfg.vocab, C.c_float(cfg.softcap),
                 _ptr(b["next"]), _ptr(b["val"]))

    def prefill(self, seq: int, ids) -> int:
        """greedy(tokenIds, startPos) for one sequence: appends the tokens at its current
        position and returns the next token id."""
        ids = np.asarray(ids, dtype=np.int32)
        T = int(ids.size)
        if T < 1 or T > self.max_rows:
            raise G4Error(-1, f"prefill of {T} tokens (1..{self.max_rows})")
        pos = int(self.seq_pos[seq].item())
        if pos + T > self.max_seq:
            raise G4Error(-6, f"KV cache capacity {self.max_seq} exceeded")
        self.buf["ids"][:T].copy_(torch.from_numpy(ids))
        rmap = G4Rows(self.seq_pos.data_ptr() + 0, seq, T, 0)
        self._forward(self.buf["ids"], T, rmap, 1, T - 1)
        call("g4_advance_positions", self.ctx.handle, _ptr(self.seq_pos), seq, 1, T)
        self.ctx.check_device()
        return int(self.buf["next"][0].item())

    def decoder(self) -> "Decoder | None":
        """The persistent decoder of this model (built on first use), or None when the model
        is batched, persistent decoding is off, or the shapes are outside its range."""
        if not self.persistent:
            return None
        if self._dec is None:
            try:
                self._dec = Decoder(self)
            except G4Error as e:
                if e.status != -5:  # only an unsupported shape falls back to the operators
                    raise
                self._dec = False
        return self._dec or None

    def decode_step(self, ids_dev: torch.Tensor | None = None, batch: int | None = None) -> torch.Tensor:
        """One greedy decode step of sequences 0..batch-1 (row b = sequence b); reads the
        current tokens from ids_dev (default: the previous step's picks) and returns the
        device tensor of the next tokens."""
        B = batch or self.max_batch
        if ids_dev is not None:
            self.buf["next"][:B].copy_(ids_dev[:B])
        dec = self.decoder() if B == 1 else None
        if dec is not None:  # the whole step in one launch: reads next[0], writes next[0] and val[0]
            dec.step(self.ctx, self.buf["next"], self.seq_pos, self.buf["next"], self.buf["val"])
            return self.buf["next"][:1]
        self.buf["ids"][:B].copy_(self.buf["next"][:B])
        # Inside a captured graph the positions and the cached history come from earlier
        # launches of the graph, so the attention may stream them before its wait.
        flags = _lib.G4_ROWS_HISTORY_READY if self._capturing else 0
        rmap = G4Rows(self.seq_pos.data_ptr(), 0, 1, 0, flags)
        self._forward(self.buf["ids"], B, rmap, B, 0)
        call("g4_advance_positions", self.ctx.handle, _ptr(self.seq_pos), 0, B, 1)
        return self.buf["next"][:B]

    def capture_decode(self, batch: int | None = None):
        """Captures one decode step (next <- argmax(model(next))) in a CUDA graph."""
        B = batch or self.max_batch
        saved = self.buf["next"][:B].clone()
        self.decode_step(batch=B)  # warm-up: sizes workspaces and sets kernel attributes
        self.ctx.sync()
        self.seq_pos[:B] -= 1      # undo the warm-up step (its K/V slot is rewritten by the replay)
        self.buf["next"][:B].copy_(saved)
        stream = torch.cuda.Stream(self.dev)
        g = torch.cuda.CUDAGraph()
        old = self.ctx.stream
        from .runtime import launch_count
        n0 = launch_count()
        with torch.cuda.stream(stream):
            self.ctx.set_stream(stream)
            self._capturing = True
            try:
                with torch.cuda.graph(g, stream=stream):
                    self.decode_step(batch=B)
            finally:
                self._capturing = False
        self.ctx.set_stream(old)
        self.graph_kernels = launch_count() - n0   # libg4w4 kernels per replayed step
        self.graph, self.graph_stream, self.graph_batch = g, stream, B
        return g

    def replay_decode(self):
        self.graph.replay()
        return self.buf["next"][: self.graph_batch]

    def fill_kv_random(self, length: int, seed: int = 0, nseq: int | None = None):
        """Synthetic context for benchmarks: K/V of positions [0, length) of every
        sequence <- random bf16 (K ~ N(0, 0.3^2), V ~ N(0, 1), the scale of normed
        keys and values), seq_pos <- length.  Decode cost does not depend on the values."""
        nseq = nseq or self.max_batch
        if length > self.max_seq:
            raise G4Error(-6, f"KV cache capacity {self.max_seq} exceeded")
        g = torch.Generator(device=self.dev).manual_seed(seed)
        cudart = C.CDLL("libcudart.so.12")
        cudart.cudaMemcpy2DAsync.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_size_t,
                                             C.c_size_t, C.c_int, C.c_void_p]
        stream = C.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)
        for Ly in self.layers:
            if Ly["spec"]["shared"]:
                continue
            hd = Ly["spec"]["hd"]
            kv = Ly["kv"]
            kp, vp = C.c_void_p(), C.c_void_p()
            call("g4_kv_buffers", kv.handle, C.byref(kp), C.byref(vp))
            pitch = self.kv_stride(kv) * hd * 2
            # (first storage row, first source row, rows) of each copy; a ring cache keeps
            # the last `ring` positions at slot p % ring, then repeats slots 0.. after the ring
            n = min(length, kv.ring) if kv.ring else length
            if kv.ring:
                s0 = (length - n) % kv.ring
                first = min(n, kv.ring - s0)
                parts = [(s0, 0, first), (0, first, n - first)]
            else:
                parts = [(0, 0, n)]
            for dst, sd in ((kp, 0.3), (vp, 1.0)):
                src = (torch.randn((nseq, n, hd), device=self.dev, generator=g) * sd).to(torch.bfloat16)
                for row, srow, cnt in parts:
                    if cnt <= 0:
                        continue
                    rc = cudart.cudaMemcpy2DAsync(dst.value + row * hd * 2, pitch, src.data_ptr() + srow * hd * 2,
                                                  n * hd * 2, cnt * hd * 2, nseq, 3, stream)
                    if rc != 0:
                        raise G4Error(-3, f"cudaMemcpy2DAsync failed ({rc})")
                if kv.ring:
                    mirror = kv.seq_rows - kv.ring
                    rc = cudart.cudaMemcpy2DAsync(dst.value + kv.ring * hd * 2, pitch, dst.value, pitch,
                                                  mirror * hd * 2, nseq, 3, stream)
                    if rc != 0:
                        raise G4Error(-3, f"cudaMemcpy2DAsync failed ({rc})")
                torch.cuda.current_stream(self.dev).synchronize()
        self.seq_pos[:nseq] = length

    def close(self):
        self.graph = None
        if self._dec:
            self._dec.close()
        self._dec = None
