"""Loading the real distribution: the W4A16 `core.safetensors` checkpoint and the PLE W4
shard set, into the weight dictionary `Gemma4Model` takes.

Tensor naming follows the reference's loader: per layer `model.language_model.layers.{i}`
with `self_attn.{q,k,v,o}_proj`, `mlp.{gate,up,down}_proj`, `per_layer_input_gate`,
`per_layer_projection` as W4A16 linears (`{base}.weight_packed` I32 [N, K/8],
`{base}.weight_scale` BF16 [N, K/32], `{base}.weight_shape` I64 [N, K];
custom-webgpu/gemma4-webgpu.js:79-95, browser-tfjs-webgl-distribution/runtime/checkpoint/
load-official-w4a16-layer.js:11-63), the six RMSNorm scales and `layer_scalar`
(gemma4-webgpu.js:102-120); top level `per_layer_model_projection`,
`per_layer_projection_norm.weight`, `norm.weight` and the tied
`embed_tokens.weight` (gemma4-webgpu.js:150-188).  KV-shared layers have no k/v
projections and no k_norm (gemma4-webgpu.js:90-93, :116).

The PLE table is the `gemma4-ple-w4-sharded-v1` format written by
tools/build_ple_w4_full.py:130-183: shards of `rows_per_shard` token rows, each file the
packed nibbles of its rows (`packed_row_bytes` each) followed by their bf16 scales
(`scale_row_bytes` each), described by manifest.json (webgpu-distribution/ple-w4/
manifest.json:12-31); token t lives in shard floor(t / rows_per_shard).

Everything here is host-side I/O; the arrays it returns go to the device through the
C ABI (W4Linear, PleW4Table, Dense) when the model is built.
"""
from __future__ import annotations

import hashlib
import json
import struct
from pathlib import Path

import numpy as np

from .model import ModelConfig

_DTYPES = {"I32": np.int32, "I64": np.int64, "BF16": np.uint16, "F32": np.float32, "U8": np.uint8,
           "I8": np.int8, "F16": np.float16}


class CheckpointError(ValueError):
    """A checkpoint or shard set that does not match what the model expects."""


class SafetensorsReader:
    """Reads tensors from a .safetensors file (8-byte little-endian header length, JSON
    header, raw little-endian data) without loading the whole file."""

    def __init__(self, path):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            n = struct.unpack("<Q", f.read(8))[0]
            self.header = json.loads(f.read(n))
        self.header.pop("__metadata__", None)
        self.data_start = 8 + n

    def has(self, name: str) -> bool:
        return name in self.header

    def info(self, name: str) -> dict:
        if name not in self.header:
            raise CheckpointError(f"{self.path.name}: no tensor {name}")
        return self.header[name]

    def read(self, name: str) -> np.ndarray:
        """The tensor as a numpy array (BF16 as its uint16 bits)."""
        info = self.info(name)
        dt = _DTYPES.get(info["dtype"])
        if dt is None:
            raise CheckpointError(f"{name}: unsupported dtype {info['dtype']}")
        start, end = info["data_offsets"]
        shape = tuple(info["shape"])
        count = int(np.prod(shape)) if shape else 1
        if end - start != count * np.dtype(dt).itemsize:
            raise CheckpointError(f"{name}: {end - start} bytes for shape {shape} {info['dtype']}")
        a = np.fromfile(self.path, dtype=np.dtype(dt).newbyteorder("<"), count=count, offset=self.data_start + start)
        return a.reshape(shape)

    def bf16_as_f32(self, name: str) -> np.ndarray:
        """reader.bf16 / readBF16Float32: bf16 bits widened to f32 (exact)."""
        bits = self.read(name)
        if self.info(name)["dtype"] != "BF16":
            raise CheckpointError(f"{name}: expected BF16, got {self.info(name)['dtype']}")
        return (bits.astype(np.uint32) << 16).view(np.float32)

    def w4_linear(self, base: str, out_dim: int, in_dim: int) -> tuple[np.ndarray, np.ndarray]:
        """loadLinear (load-official-w4a16-layer.js:11-39): packed I32 [N, K/8] and the
        bf16 scale bits [N, K/32], after checking `{base}.weight_shape` = [N, K]."""
        packed = self.read(f"{base}.weight_packed")
        scales = self.read(f"{base}.weight_scale")
        if self.has(f"{base}.weight_shape"):
            shape = [int(v) for v in self.read(f"{base}.weight_shape").reshape(-1)]
            if shape != [out_dim, in_dim]:
                raise CheckpointError(f"{base}: packed checkpoint {shape} != Linear [{out_dim}, {in_dim}]")
        if packed.dtype != np.int32 or packed.shape != (out_dim, in_dim // 8):
            raise CheckpointError(f"{base}.weight_packed: {packed.dtype} {packed.shape}, expected int32 "
                                  f"[{out_dim}, {in_dim // 8}]")
        if self.info(f"{base}.weight_scale")["dtype"] != "BF16" or scales.shape[0] != out_dim or \
                in_dim % scales.shape[1] != 0:
            raise CheckpointError(f"{base}.weight_scale: {self.info(f'{base}.weight_scale')['dtype']} {scales.shape}")
        if in_dim // scales.shape[1] != 32:
            raise CheckpointError(f"{base}: group size {in_dim // scales.shape[1]} (32 supported)")
        return packed, scales

    def scalar(self, name: str) -> float:
        """reader.scalarBF16 (gemma4-webgpu.js:118)."""
        return float(self.bf16_as_f32(name).reshape(-1)[0])


def layer_names(cfg: ModelConfig, i: int) -> dict:
    """linearsForLayer (gemma4-webgpu.js:79-95) and the norms of loadLayer (:109-117)."""
    root = f"model.language_model.layers.{i}"
    s = cfg.spec(i)
    names = {
        "q": f"{root}.self_attn.q_proj", "o": f"{root}.self_attn.o_proj",
        "gate": f"{root}.mlp.gate_proj", "up": f"{root}.mlp.up_proj", "down": f"{root}.mlp.down_proj",
        "pg": f"{root}.per_layer_input_gate", "pp": f"{root}.per_layer_projection",
        "n_in": f"{root}.input_layernorm.weight", "n_pa": f"{root}.post_attention_layernorm.weight",
        "n_pf": f"{root}.pre_feedforward_layernorm.weight", "n_pff": f"{root}.post_feedforward_layernorm.weight",
        "n_pple": f"{root}.post_per_layer_input_norm.weight", "qn": f"{root}.self_attn.q_norm.weight",
        "skip": f"{root}.layer_scalar",
    }
    if not s["shared"]:
        names.update(k=f"{root}.self_attn.k_proj", v=f"{root}.self_attn.v_proj",
                     kn=f"{root}.self_attn.k_norm.weight")
    return names


def tensor_names(cfg: ModelConfig) -> list[str]:
    """Every tensor the loader reads: the W4A16 triples (packed, scale, shape) of each
    linear, the norms, the layer scalars and the top-level tensors."""
    names = []
    for i in range(cfg.layers):
        for key, base in layer_names(cfg, i).items():
            if key in ("q", "k", "v", "o", "gate", "up", "down", "pg", "pp"):
                names += [f"{base}.weight_packed", f"{base}.weight_scale", f"{base}.weight_shape"]
            else:
                names.append(base)
    top = TOP["top"]
    names += [f"{top}.weight_packed", f"{top}.weight_scale", f"{top}.weight_shape"]
    names += [TOP["ple_norm"], TOP["final_norm"], TOP["embed"]]
    return names


TOP = {"top": "model.language_model.per_layer_model_projection",
       "ple_norm": "model.language_model.per_layer_projection_norm.weight",
       "final_norm": "model.language_model.norm.weight",
       "embed": "model.language_model.embed_tokens.weight"}


def load_weights(reader: SafetensorsReader, cfg: ModelConfig, ple: "PleShardSet | None" = None) -> dict:
    """Gemma4WebGPU.load (gemma4-webgpu.js:150-188) into `Gemma4Model`'s weight dictionary:
    q/k/v rows concatenated into one linear, gate/up rows into another (the same bits,
    one launch each), norms widened to f32, the tied embedding as bf16 bits, and the PLE
    table from the shard set when one is given."""
    H, P, L = cfg.hidden, cfg.ple_dim, cfg.layers
    w = {"layers": []}
    for i in range(L):
        s = cfg.spec(i)
        hd, inter = s["hd"], s["inter"]
        n = layer_names(cfg, i)
        lw = {}
        parts = [reader.w4_linear(n["q"], cfg.heads * hd, H)]
        if not s["shared"]:
            parts += [reader.w4_linear(n["k"], hd, H), reader.w4_linear(n["v"], hd, H)]
        lw["qkv"] = (np.concatenate([p for p, _ in parts]), np.concatenate([sc for _, sc in parts]))
        lw["o"] = reader.w4_linear(n["o"], H, cfg.heads * hd)
        g, u = reader.w4_linear(n["gate"], inter, H), reader.w4_linear(n["up"], inter, H)
        lw["gu"] = (np.concatenate([g[0], u[0]]), np.concatenate([g[1], u[1]]))
        lw["down"] = reader.w4_linear(n["down"], H, inter)
        lw["pg"] = reader.w4_linear(n["pg"], P, H)
        lw["pp"] = reader.w4_linear(n["pp"], H, P)
        for key, width in (("n_in", H), ("n_pa", H), ("n_pf", H), ("n_pff", H), ("n_pple", H), ("qn", hd)):
            lw[key] = _norm(reader, n[key], width)
        # a KV-shared layer normalises no k of its own (gemma4-webgpu.js:116)
        lw["kn"] = _norm(reader, n["kn"], hd) if "kn" in n else np.ones(hd, np.float32)
        lw["skip"] = reader.scalar(n["skip"])
        w["layers"].append(lw)
    w["top"] = reader.w4_linear(TOP["top"], L * P, H)
    w["ple_norm"] = _norm(reader, TOP["ple_norm"], P)
    w["final_norm"] = _norm(reader, TOP["final_norm"], H)
    emb = reader.read(TOP["embed"])
    if reader.info(TOP["embed"])["dtype"] != "BF16" or emb.shape != (cfg.vocab, H):
        raise CheckpointError(f"{TOP['embed']}: {reader.info(TOP['embed'])['dtype']} {emb.shape}, expected BF16 "
                              f"[{cfg.vocab}, {H}]")
    w["embed"] = emb
    if ple is not None:
        if ple.vocab != cfg.vocab or ple.width != L * P:
            raise CheckpointError(f"PLE shards [{ple.vocab}, {ple.width}] != model [{cfg.vocab}, {L * P}]")
        w["ple_packed"], w["ple_scales"] = ple.load_all()
    return w


def _norm(reader: SafetensorsReader, name: str, width: int) -> np.ndarray:
    a = reader.bf16_as_f32(name).reshape(-1)
    if a.shape != (width,):
        raise CheckpointError(f"{name}: expected [{width}], got {list(a.shape)}")
    return a.astype(np.float32)


class PleShardSet:
    """The `gemma4-ple-w4-sharded-v1` PLE table on disk (manifest + shard files)."""

    FORMAT = "gemma4-ple-w4-sharded-v1"

    def __init__(self, manifest_path, verify_hashes: bool = False):
        self.manifest_path = Path(manifest_path)
        m = json.loads(self.manifest_path.read_text())
        if m.get("format") != self.FORMAT:
            raise CheckpointError(f"PLE manifest format {m.get('format')!r} (expected {self.FORMAT})")
        if not m.get("complete", False):
            raise CheckpointError("PLE manifest is not complete (an interrupted build)")
        q, lay = m["quantization"], m["layout"]
        self.vocab, self.width = int(m["vocab_size"]), int(m["width"])
        self.group = int(q["group_size"])
        if (q["bits"], q["qmin"], q["qmax"], q["scale_dtype"], q["nibble_order"], q["signed_encoding"]) != \
                (4, -7, 7, "BF16", "low_first", "two_complement_nibble") or q.get("zero_point"):
            raise CheckpointError(f"PLE quantisation {q} is not the W4 format the gather decodes")
        if lay["kind"] != "row_sharded_packed_then_scales":
            raise CheckpointError(f"PLE layout {lay['kind']!r}")
        self.rows_per_shard = int(lay["rows_per_shard"])
        self.packed_row, self.scale_row = int(lay["packed_row_bytes"]), int(lay["scale_row_bytes"])
        if self.packed_row != self.width // 2 or self.scale_row != self.width // self.group * 2:
            raise CheckpointError(f"PLE row bytes {self.packed_row}/{self.scale_row} for width {self.width}")
        self.shards = sorted(m["shards"], key=lambda s: s["index"])
        row = 0
        for s in self.shards:
            rows = int(s["rows"])
            if int(s["row_start"]) != row or int(s["row_end"]) != row + rows or \
                    int(s["packed_offset"]) != 0 or int(s["packed_bytes"]) != rows * self.packed_row or \
                    int(s["scales_offset"]) != rows * self.packed_row or int(s["scales_bytes"]) != rows * self.scale_row:
                raise CheckpointError(f"PLE shard {s['index']}: inconsistent extents {s}")
            row += rows
        if row != self.vocab:
            raise CheckpointError(f"PLE shards cover {row} rows of {self.vocab}")
        self.verify_hashes = verify_hashes
        self.verification_rows = [int(r) for r in m.get("verification_rows", [])]

    def shard_of(self, token: int) -> int:
        """token_to_shard: floor(token_id / rows_per_shard)."""
        if not 0 <= token < self.vocab:
            raise CheckpointError(f"PLE token {token} out of range [0, {self.vocab})")
        return token // self.rows_per_shard

    def _shard_bytes(self, s: dict) -> bytes:
        path = self.manifest_path.parent / s["file"]
        data = path.read_bytes()
        if len(data) != int(s["bytes"]):
            raise CheckpointError(f"{s['file']}: {len(data)} bytes, manifest says {s['bytes']}")
        if self.verify_hashes and s.get("sha256") and hashlib.sha256(data).hexdigest() != s["sha256"]:
            raise CheckpointError(f"{s['file']}: sha256 mismatch")
        return data

    def load_all(self) -> tuple[np.ndarray, np.ndarray]:
        """The whole table as packed nibbles u8 [vocab, width/2] and bf16 scale bits u16
        [vocab, width/group] (the arrays PleW4Table / g4_ple_table_create take)."""
        packed = np.empty((self.vocab, self.packed_row), np.uint8)
        scales = np.empty((self.vocab, self.width // self.group), np.uint16)
        for s in self.shards:
            data = self._shard_bytes(s)
            r0, rows = int(s["row_start"]), int(s["rows"])
            pb = rows * self.packed_row
            packed[r0:r0 + rows] = np.frombuffer(data, np.uint8, pb).reshape(rows, self.packed_row)
            scales[r0:r0 + rows] = np.frombuffer(data, "<u2", rows * self.scale_row // 2, pb).reshape(rows, -1)
        return packed, scales

    def read_rows(self, ids) -> tuple[np.ndarray, np.ndarray]:
        """The packed and scale rows of the given tokens, read from their shards only."""
        ids = np.asarray(ids, np.int64).reshape(-1)
        packed = np.empty((ids.size, self.packed_row), np.uint8)
        scales = np.empty((ids.size, self.width // self.group), np.uint16)
        cache: dict[int, bytes] = {}
        for j, t in enumerate(ids):
            si = self.shard_of(int(t))
            s = self.shards[si]
            if si not in cache:
                cache[si] = self._shard_bytes(s)
            data, local, rows = cache[si], int(t) - int(s["row_start"]), int(s["rows"])
            packed[j] = np.frombuffer(data, np.uint8, self.packed_row, local * self.packed_row)
            scales[j] = np.frombuffer(data, "<u2", self.scale_row // 2, rows * self.packed_row + local * self.scale_row)
        return packed, scales


def load_model(ctx, cfg: ModelConfig, checkpoint, ple_manifest, **model_kw):
    """Gemma4WebGPU + load() over libg4w4: the model built from the distribution's files."""
    from .model import Gemma4Model
    w = load_weights(SafetensorsReader(checkpoint), cfg, PleShardSet(ple_manifest))
    return Gemma4Model(ctx, cfg, w, **model_kw)
