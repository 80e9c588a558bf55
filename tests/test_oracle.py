"""CPU tests: the oracle against the reference-generated golden vectors and its numpy twin."""
import numpy as np
import pytest

from conftest import golden, max_rel


def test_rne_matches_reference_helper(oracle):
    g = golden("rne_golden.npz")
    assert np.array_equal(oracle.f32_to_bf16_bits(g["f32"]), g["bf16"])
    L = oracle.lib()
    c = np.array([L.g4o_f32_to_bf16_bits(float(v)) for v in g["f32"][:64]], np.uint16)
    assert np.array_equal(c, g["bf16"][:64])


def test_ple_geometry_matches_manifest():
    g = golden("ple_w4_golden.npz")
    assert int(g["width"]) == 8960 and int(g["group"]) == 32
    assert int(g["packed_row_bytes"]) == int(g["width"]) // 2
    assert int(g["scale_row_bytes"]) == int(g["width"]) // int(g["group"]) * 2
    assert int(g["vocab"]) == 262144 and int(g["qmin"]) == -7 and int(g["qmax"]) == 7


def test_ple_oracle_decodes_reference_quantiser_output(oracle, npo):
    g = golden("ple_w4_golden.npz")
    ids = g["ids"]
    f32 = oracle.ple_read_rows(g["packed"], g["scales"], ids)
    assert np.array_equal(f32.view(np.uint32), g["expected_f32"][ids].view(np.uint32))
    b16 = oracle.ple_read_rows(g["packed"], g["scales"], ids, bf16=True)
    assert np.array_equal(b16, g["expected_bf16"][ids])
    assert np.array_equal(npo.ple_read_rows(g["packed"], g["scales"], ids).view(np.uint32),
                          g["expected_f32"][ids].view(np.uint32))
    # multi-threaded path gives the same bytes
    assert np.array_equal(oracle.ple_read_rows(g["packed"], g["scales"], ids, nthreads=3), f32)


def test_ple_oracle_rejects_out_of_range(oracle):
    g = golden("ple_w4_golden.npz")
    with pytest.raises(oracle.OracleError):
        oracle.ple_read_rows(g["packed"], g["scales"], np.array([0, 24], np.int32))
    with pytest.raises(oracle.OracleError):
        oracle.ple_read_rows(g["packed"], g["scales"], np.array([-1], np.int32))


def test_linear_known_answers(oracle, npo):
    g = golden("linear_w4_golden.npz")
    out = oracle.dequant_w4a16_rows(g["packed"], g["scales"])
    assert np.array_equal(out, g["expected_f32"])
    assert np.array_equal(npo.dequant_w4a16(g["packed"], g["scales"]), g["expected_f32"])
    assert np.array_equal(npo.unpack_linear_q(g["packed"]), g["q"])


def test_linear_format_matches_compressed_tensors(oracle, npo):
    """The pack-quantized format as its producer writes it (compressed-tensors 0.15.0.1:
    pack_to_int32 and dequantize, tests/golden/make_golden.py --compressed-tensors): the
    oracle unpacks the library's words to its q and dequantises them to its bf16 weights,
    bit for bit (extreme q, a zero group, subnormal-adjacent and overflowing scales)."""
    g = golden("linear_w4_ct_golden.npz")
    assert np.array_equal(npo.unpack_linear_q(g["packed"]), g["q"])
    f32 = oracle.dequant_w4a16_rows(g["packed"], g["scales"])
    assert np.array_equal(oracle.f32_to_bf16_bits(f32), g["expected_bf16"])
    with np.errstate(over="ignore"):  # the 3e38 scales overflow to inf on purpose
        assert np.array_equal(npo.dequant_w4a16(g["packed"], g["scales"]), f32)


@pytest.mark.parametrize("M,K,N", [(1, 64, 40), (3, 96, 24), (5, 256, 300)])
def test_linear_oracle_vs_numpy(oracle, npo, M, K, N):
    rng = np.random.default_rng(M * 1000 + K)
    packed = rng.integers(0, 2**32, size=(N, K // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    scales = oracle.f32_to_bf16_bits(np.abs(rng.normal(0, 0.02, (N, K // 32))).astype(np.float32))
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = oracle.linear_w4a16(x, packed, scales)
    ref = npo.linear_w4a16(x, packed, scales)
    assert max_rel(y, ref) < 1e-5
    assert np.array_equal(oracle.linear_w4a16(x, packed, scales, nthreads=2), y)
    # dequant rows window
    part = oracle.dequant_w4a16_rows(packed, scales, row_start=3, row_count=5)
    assert np.array_equal(part, npo.dequant_w4a16(packed, scales)[3:8])


@pytest.mark.parametrize("rows,keylen,qpos0,sliding,window", [
    (1, 1, 0, False, 512), (1, 600, 599, True, 512), (4, 40, 36, False, 512), (3, 30, 27, True, 8),
])
def test_attention_oracle_vs_numpy(oracle, npo, rows, keylen, qpos0, sliding, window):
    rng = np.random.default_rng(keylen)
    q = rng.standard_normal((rows, 8, 64)).astype(np.float32) * 0.3
    k = rng.standard_normal((keylen, 64)).astype(np.float32)
    v = rng.standard_normal((keylen, 64)).astype(np.float32)
    a = oracle.attention(q, k, v, qpos0, sliding, window)
    b = npo.attention(q, k, v, qpos0, sliding, window)
    assert max_rel(a, b) < 1e-5
