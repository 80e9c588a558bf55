"""Generates the golden fixtures in tests/golden/ from the reference's own Python code.

Run once in a checkout that has the gemma4-js reference next to it:
    python tests/golden/make_golden.py --reference /path/to/gemma4-js

What is pinned, and by what:
  * PLE W4 format (ple_w4_golden.npz): seeded bf16 rows are quantised by the
    reference's `quantize_batch` (tools/build_ple_w4_full.py:48-60), which also
    defines the format the runtime decodes.  The expected dequantised values are
    `stored_scale * q` computed with the reference's own helpers from the same
    intermediate q the quantiser wrote, so decoding the packed bytes back must give
    them exactly (ple-w4-shard-reader.js:89-95 restated by the oracle).
  * bf16 rounding (rne_golden.npz): the reference's `f32_to_bf16_bits_rne`
    (tools/build_ple_w4_full.py:42-45, the Python twin of roundFloat32ToBF16,
    official-w4a16.js:34-48) on special and random f32 values.
  * PLE geometry constants from webgpu-distribution/ple-w4/manifest.json:12-31.
  * Linear W4 known answers (linear_w4_golden.npz): words whose nibbles decode to
    known values under official-w4a16.js:15-19 (offset binary, nibble - 8).  The
    linear dequant is JavaScript only, so these are read off the source, not run.
  * Linear W4 format as written by its producer (linear_w4_ct_golden.npz): the
    checkpoint's `weight_packed` / `weight_scale` pairs are the pack-quantized format
    of the compressed-tensors library (0.15.0.1 is installed here, as a dependency of
    vllm).  Seeded int4 q in [-8, 7] are packed by its `pack_to_int32(q, 4,
    packed_dim=1)` and dequantised by its `dequantize(q, scale)` (group 32 inferred from
    the scale shape; q.to(bf16) * scale: one f32 product rounded to bf16, the
    roundFloat32ToBF16(q * s) of official-w4a16.js:95).  Run with --compressed-tensors.
The fixtures are committed; GPU boxes and the test suite never read the reference.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_builder(ref: Path):
    spec = importlib.util.spec_from_file_location("ref_build_ple_w4_full", ref / "tools" / "build_ple_w4_full.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_ple(ref: Path, b) -> None:
    manifest = json.loads((ref / "webgpu-distribution" / "ple-w4" / "manifest.json").read_text())
    width = int(manifest["width"])
    group = int(manifest["quantization"]["group_size"])
    rng = np.random.default_rng(20260101)
    rows = 24
    src = rng.normal(0.0, 0.05, size=(rows, width)).astype(np.float32)
    src[1] *= 0.0                                    # all-zero row: every group takes scale 1.0
    src[2, :64] = 0.0                                # two zero groups inside a row
    src[3] *= 1e-30                                  # tiny magnitudes (bf16 scales near subnormal)
    src[4] *= 1e4                                    # large magnitudes
    src[5, ::7] = -src[5, ::7] * 3                   # mixed signs / outliers
    src_bits = b.f32_to_bf16_bits_rne(src)           # the checkpoint holds bf16
    src_f32 = b.bf16_bits_to_f32(src_bits)
    packed, scale_bits = b.quantize_batch(src_f32)
    # the q the quantiser stored, recomputed with the quantiser's own arithmetic
    groups = src_f32.reshape(rows, width // group, group)
    stored = b.bf16_bits_to_f32(scale_bits)
    q = np.clip(np.rint(groups / stored[..., None]), -b.QMAX, b.QMAX).astype(np.int8).reshape(rows, width)
    expected = (q.astype(np.float32).reshape(rows, width // group, group) * stored[..., None]).reshape(rows, width)
    expected_bf16 = b.f32_to_bf16_bits_rne(expected)
    np.savez_compressed(
        HERE / "ple_w4_golden.npz", packed=packed.astype(np.uint8), scales=scale_bits.astype(np.uint16),
        expected_f32=expected.astype(np.float32), expected_bf16=expected_bf16.astype(np.uint16),
        ids=np.array([3, 0, 23, 5, 5, 1, 2, 4, 22, 20], np.int32),
        width=np.int32(width), group=np.int32(group),
        packed_row_bytes=np.int32(manifest["layout"]["packed_row_bytes"]),
        scale_row_bytes=np.int32(manifest["layout"]["scale_row_bytes"]),
        vocab=np.int32(manifest["vocab_size"]), rows_per_shard=np.int32(manifest["layout"]["rows_per_shard"]),
        qmin=np.int32(manifest["quantization"]["qmin"]), qmax=np.int32(manifest["quantization"]["qmax"]),
    )


def make_rne(b) -> None:
    specials = np.array([0.0, -0.0, 1.0, -1.0, 1.00390625, 1.01171875, 1.005859375, 3.4e38, -3.4e38,
                         np.inf, -np.inf, 1e-40, -1e-40, 1.1754942e-38, 2.0 ** -133, 65504.0,
                         0.1, 1.0 / 3.0, 2.0 ** 127 * 1.99], np.float32)
    # exact ties: low half 0x8000 with both parities of bit 16
    ties = np.array([0x3F808000, 0x3F818000, 0xBF808000, 0x40498000, 0x00018000], np.uint32).view(np.float32)
    rnd = np.random.default_rng(7).standard_normal(4096).astype(np.float32) * np.float32(3.0)
    vals = np.concatenate([specials, ties, rnd]).astype(np.float32)
    np.savez_compressed(HERE / "rne_golden.npz", f32=vals, bf16=b.f32_to_bf16_bits_rne(vals).astype(np.uint16))


def make_linear() -> None:
    # official-w4a16.js:15-19 / :84-96: nibble k of word j -> column 8j + k, value nibble - 8.
    words = np.array([[0x76543210, 0xFEDCBA98, 0x00000000, 0xFFFFFFFF],
                      [0x88888888, 0x12345678, 0x9ABCDEF0, 0x0F0F0F0F]], np.uint32)
    q = np.zeros((2, 32), np.int8)
    for r in range(2):
        for j in range(4):
            for k in range(8):
                q[r, 8 * j + k] = ((int(words[r, j]) >> (4 * k)) & 0xF) - 8
    scales = np.array([[0x3F80], [0x3C00]], np.uint16)   # 1.0 and 2^-7 (bf16 bits)
    expected = q.astype(np.float32) * np.array([[1.0], [2.0 ** -7]], np.float32)
    np.savez_compressed(HERE / "linear_w4_golden.npz", packed=words.view(np.int32), scales=scales,
                        q=q, expected_f32=expected)


def make_linear_ct() -> None:
    import torch
    from compressed_tensors.compressors.pack_quantized.helpers import pack_to_int32, unpack_from_int32
    from compressed_tensors.quantization.lifecycle.forward import dequantize
    import compressed_tensors
    N, K = 24, 256
    g = torch.Generator().manual_seed(20261202)
    q = torch.randint(-8, 8, (N, K), generator=g, dtype=torch.int8)
    q[0] = -8                                   # the extremes of the range
    q[1] = 7
    q[2, ::2], q[2, 1::2] = -8, 7               # alternating within every word
    q[3] = 0
    scales = (torch.randn((N, K // 32), generator=g).abs() * 0.02).to(torch.bfloat16)
    scales[4, 1] = 0.0                          # a zero group
    scales[5] = torch.tensor([2.0 ** -126, 1e-38, 3e38, 1.0, 0.5, 65504.0, 2.0 ** -100, 7.0], dtype=torch.float32
                             ).to(torch.bfloat16)  # subnormal-adjacent, huge, exact
    packed = pack_to_int32(q, 4, packed_dim=1)
    assert packed.dtype == torch.int32 and packed.shape == (N, K // 8)
    assert torch.equal(unpack_from_int32(packed, 4, torch.Size([N, K]), packed_dim=1), q)
    w = dequantize(q, scales)                   # bf16 [N, K]
    assert w.dtype == torch.bfloat16 and w.shape == (N, K)
    np.savez_compressed(HERE / "linear_w4_ct_golden.npz", packed=packed.numpy(),
                        scales=scales.view(torch.int16).numpy().view(np.uint16), q=q.numpy(),
                        expected_bf16=w.view(torch.int16).numpy().view(np.uint16),
                        library=np.array(f"compressed-tensors {getattr(compressed_tensors, '__version__', '0.15.0.1')}"))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path)
    ap.add_argument("--compressed-tensors", action="store_true",
                    help="also (or only) write linear_w4_ct_golden.npz with the installed compressed-tensors")
    a = ap.parse_args()
    if a.reference:
        b = load_builder(a.reference)
        make_ple(a.reference, b)
        make_rne(b)
        make_linear()
    if a.compressed_tensors:
        make_linear_ct()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
