"""CPU tests of the distribution loader (gemma4-js_b200/checkpoint.py): a checkpoint in the
reference's tensor naming and a PLE shard set in its on-disk layout are written from seeded
random weights, then read back into exactly the weight dictionary the model takes."""
import hashlib
import importlib
import json
import struct

import numpy as np
import pytest

ckpt = importlib.import_module("gemma4-js_b200.checkpoint")
model = importlib.import_module("gemma4-js_b200.model")

CFG = model.ModelConfig.reference_spec().small(hidden=512, layers=7, vocab=512, intermediate=1024,
                                               intermediate_late=2048, first_shared=5, window=16)


def _bf16(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def write_safetensors(path, tensors):
    """tensors: name -> (dtype string, array); little-endian, no padding."""
    header, blobs, off = {}, [], 0
    for name, (dt, a) in tensors.items():
        b = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(np.shape(a)), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_checkpoint(path, cfg, w):
    t = {}

    def lin(base, packed, scales):
        t[f"{base}.weight_packed"] = ("I32", packed)
        t[f"{base}.weight_scale"] = ("BF16", scales)
        t[f"{base}.weight_shape"] = ("I64", np.array([packed.shape[0], packed.shape[1] * 8], np.int64))

    H = cfg.hidden
    for i, lw in enumerate(w["layers"]):
        s, n = cfg.spec(i), ckpt.layer_names(cfg, i)
        hd, inter = s["hd"], s["inter"]
        qp, qs = lw["qkv"]
        nq = cfg.heads * hd
        lin(n["q"], qp[:nq], qs[:nq])
        if not s["shared"]:
            lin(n["k"], qp[nq:nq + hd], qs[nq:nq + hd])
            lin(n["v"], qp[nq + hd:], qs[nq + hd:])
            t[n["kn"]] = ("BF16", _bf16(lw["kn"]))
        lin(n["o"], *lw["o"])
        lin(n["gate"], lw["gu"][0][:inter], lw["gu"][1][:inter])
        lin(n["up"], lw["gu"][0][inter:], lw["gu"][1][inter:])
        lin(n["down"], *lw["down"])
        lin(n["pg"], *lw["pg"])
        lin(n["pp"], *lw["pp"])
        for key in ("n_in", "n_pa", "n_pf", "n_pff", "n_pple", "qn"):
            t[n[key]] = ("BF16", _bf16(lw[key]))
        t[n["skip"]] = ("BF16", _bf16(np.array([lw["skip"]], np.float32)))
    lin(ckpt.TOP["top"], *w["top"])
    t[ckpt.TOP["ple_norm"]] = ("BF16", _bf16(w["ple_norm"]))
    t[ckpt.TOP["final_norm"]] = ("BF16", _bf16(w["final_norm"]))
    t[ckpt.TOP["embed"]] = ("BF16", w["embed"])
    assert H == w["embed"].shape[1]
    write_safetensors(path, t)


def write_ple_shards(dirpath, packed, scales, rows_per_shard, group=32):
    vocab, width = packed.shape[0], packed.shape[1] * 2
    shards, n = [], (vocab + rows_per_shard - 1) // rows_per_shard
    for si in range(n):
        r0, r1 = si * rows_per_shard, min(vocab, (si + 1) * rows_per_shard)
        data = packed[r0:r1].tobytes() + scales[r0:r1].astype("<u2").tobytes()
        name = f"ple-{si:05d}-of-{n:05d}.bin"
        (dirpath / name).write_bytes(data)
        shards.append({"index": si, "file": name, "row_start": r0, "row_end": r1, "rows": r1 - r0,
                       "packed_offset": 0, "packed_bytes": (r1 - r0) * width // 2,
                       "scales_offset": (r1 - r0) * width // 2, "scales_bytes": (r1 - r0) * width // group * 2,
                       "bytes": len(data), "sha256": hashlib.sha256(data).hexdigest()})
    manifest = {"format": "gemma4-ple-w4-sharded-v1", "version": 1, "complete": True,
                "tensor": "model.language_model.embed_tokens_per_layer.weight", "shape": [vocab, width],
                "source_dtype": "BF16", "width": width, "vocab_size": vocab,
                "quantization": {"bits": 4, "signed": True, "symmetric": True, "qmin": -7, "qmax": 7,
                                 "group_size": group, "scale_dtype": "BF16", "zero_point": False,
                                 "nibble_order": "low_first", "signed_encoding": "two_complement_nibble"},
                "layout": {"kind": "row_sharded_packed_then_scales", "rows_per_shard": rows_per_shard,
                           "packed_row_bytes": width // 2, "scale_row_bytes": width // group * 2,
                           "token_to_shard": "floor(token_id / rows_per_shard)"},
                "shards": shards, "verification_rows": [0, 3, vocab - 1]}
    path = dirpath / "manifest.json"
    path.write_text(json.dumps(manifest))
    return path


@pytest.fixture(scope="module")
def dist(tmp_path_factory):
    d = tmp_path_factory.mktemp("dist")
    w = model.random_weights(CFG, seed=5)
    write_checkpoint(d / "core.safetensors", CFG, w)
    manifest = write_ple_shards(d, w["ple_packed"], w["ple_scales"], rows_per_shard=200)
    return d, w, manifest


def test_checkpoint_round_trip(dist):
    d, w, manifest = dist
    got = ckpt.load_weights(ckpt.SafetensorsReader(d / "core.safetensors"), CFG, ckpt.PleShardSet(manifest, True))
    for i, (a, b) in enumerate(zip(w["layers"], got["layers"])):
        for key in ("qkv", "o", "gu", "down", "pg", "pp"):
            assert np.array_equal(a[key][0], b[key][0]) and np.array_equal(a[key][1], b[key][1]), (i, key)
        for key in ("n_in", "n_pa", "n_pf", "n_pff", "n_pple", "qn"):
            assert np.array_equal(_f32(_bf16(a[key])), b[key]), (i, key)
        if CFG.spec(i)["shared"]:
            assert np.array_equal(b["kn"], np.ones_like(b["kn"]))
        else:
            assert np.array_equal(_f32(_bf16(a["kn"])), b["kn"])
        assert b["skip"] == float(_f32(_bf16(np.array([a["skip"]], np.float32)))[0])
    for key in ("top",):
        assert np.array_equal(w[key][0], got[key][0]) and np.array_equal(w[key][1], got[key][1])
    assert np.array_equal(w["embed"], got["embed"])
    assert np.array_equal(w["ple_packed"], got["ple_packed"]) and np.array_equal(w["ple_scales"], got["ple_scales"])


def test_ple_shards_rows_and_errors(dist, tmp_path):
    d, w, manifest = dist
    ple = ckpt.PleShardSet(manifest, verify_hashes=True)
    assert (ple.vocab, ple.width, ple.rows_per_shard) == (CFG.vocab, CFG.layers * CFG.ple_dim, 200)
    assert [ple.shard_of(t) for t in (0, 199, 200, 511)] == [0, 0, 1, 2]
    ids = [511, 0, 200, 199, 7, 7]
    p, s = ple.read_rows(ids)
    assert np.array_equal(p, w["ple_packed"][ids]) and np.array_equal(s, w["ple_scales"][ids])
    with pytest.raises(ckpt.CheckpointError):
        ple.shard_of(512)
    # a corrupted shard byte is caught by the manifest's sha256
    m = json.loads(manifest.read_text())
    bad = tmp_path / "bad"
    bad.mkdir()
    for s in m["shards"]:
        data = bytearray((d / s["file"]).read_bytes())
        if s["index"] == 1:
            data[10] ^= 0xFF
        (bad / s["file"]).write_bytes(bytes(data))
    (bad / "manifest.json").write_text(json.dumps(m))
    with pytest.raises(ckpt.CheckpointError, match="sha256"):
        ckpt.PleShardSet(bad / "manifest.json", verify_hashes=True).load_all()
    m2 = dict(m, complete=False)
    (bad / "manifest.json").write_text(json.dumps(m2))
    with pytest.raises(ckpt.CheckpointError, match="not complete"):
        ckpt.PleShardSet(bad / "manifest.json")


def test_checkpoint_shape_mismatch_is_an_error(dist, tmp_path):
    d, w, _ = dist
    r = ckpt.SafetensorsReader(d / "core.safetensors")
    base = ckpt.layer_names(CFG, 0)["o"]
    with pytest.raises(ckpt.CheckpointError, match="packed checkpoint"):
        r.w4_linear(base, CFG.hidden + 8, CFG.heads * CFG.spec(0)["hd"])
    with pytest.raises(ckpt.CheckpointError, match="no tensor"):
        r.read("model.language_model.layers.99.self_attn.q_proj.weight_packed")


def test_reference_checkpoint_tensor_count():
    """The names the loader reads for the checkpoint's own spec (35 layers, KV sharing from
    layer 15) are distinct and exactly as many as the distribution's core.safetensors
    holds: 1091 tensors (webgpu-distribution/core.safetensors.manifest.json, tensor_count)."""
    names = ckpt.tensor_names(model.ModelConfig.reference_spec())
    assert len(names) == len(set(names)) == 1091
