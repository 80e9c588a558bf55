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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    a = ap.parse_args()
    b = load_builder(a.reference)
    make_ple(a.reference, b)
    make_rne(b)
    make_linear()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
