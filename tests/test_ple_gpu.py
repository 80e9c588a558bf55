"""PLE W4 gather-dequant on the GPU through the C ABI, bit-exact against the oracle."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.cpu().view(torch.int32 if t.dtype == torch.float32 else torch.int16).numpy()


def test_golden_rows_bit_exact(rt, ctx):
    g = golden("ple_w4_golden.npz")
    tab = rt.PleW4Table(ctx, g["packed"], g["scales"])
    ids = g["ids"]
    out32 = tab.rows_to_gpu(ids, torch.float32)
    out16 = tab.rows_to_gpu(ids, torch.bfloat16)
    ctx.check_device()
    assert np.array_equal(_bits(out32), g["expected_f32"][ids].view(np.int32))
    assert np.array_equal(_bits(out16), g["expected_bf16"][ids].view(np.int16))


@pytest.mark.parametrize("T", [1, 7, 1000])
def test_random_table_bit_exact(rt, ctx, oracle, T):
    rng = np.random.default_rng(T)
    vocab, width = 3000, 8960
    q = rng.integers(-7, 8, size=(vocab, width), dtype=np.int8)
    nib = (q.astype(np.int16) & 0xF).astype(np.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    scales = oracle.f32_to_bf16_bits(np.abs(rng.normal(0, 0.05, (vocab, width // 32))).astype(np.float32))
    tab = rt.PleW4Table(ctx, packed, scales)
    ids = rng.integers(0, vocab, size=T).astype(np.int32)
    ids[: min(T, 3)] = ids[0]  # duplicates
    for dt, bf in ((torch.float32, False), (torch.bfloat16, True)):
        out = tab.rows_to_gpu(ids, dt)
        ref = oracle.ple_read_rows(packed, scales, ids, bf16=bf)
        assert np.array_equal(_bits(out), ref.view(np.int32 if not bf else np.int16))
    # device-resident ids give the same rows
    out_dev = tab.rows_to_gpu(torch.from_numpy(ids).cuda(), torch.bfloat16)
    assert torch.equal(out_dev, tab.rows_to_gpu(ids, torch.bfloat16))
    ctx.check_device()


def test_special_scale_values(rt, ctx, oracle):
    # subnormal, largest finite, infinity and NaN scales; every nibble value
    vocab, width = 4, 64
    packed = np.tile(np.arange(256, dtype=np.uint8)[:32], (vocab, 1))
    scales = np.array([[0x0001, 0x7F7F], [0x8001, 0x7F80], [0x7FC0, 0x0000], [0x3F80, 0xBF80]], np.uint16)
    tab = rt.PleW4Table(ctx, packed, scales, width=width)
    ids = np.arange(vocab, dtype=np.int32)
    f32 = tab.rows_to_gpu(ids, torch.float32).cpu().numpy()
    ref32 = oracle.ple_read_rows(packed, scales, ids)
    nan = np.isnan(ref32)
    assert np.array_equal(np.isnan(f32), nan)
    assert np.array_equal(f32[~nan].view(np.uint32), ref32[~nan].view(np.uint32))
    b16 = _bits(tab.rows_to_gpu(ids, torch.bfloat16)).view(np.uint16)
    ref16 = oracle.ple_read_rows(packed, scales, ids, bf16=True)
    nan16 = ((ref16 & 0x7F80) == 0x7F80) & ((ref16 & 0x7F) != 0)
    assert np.array_equal(((b16 & 0x7F80) == 0x7F80) & ((b16 & 0x7F) != 0), nan16)
    assert np.array_equal(b16[~nan16], ref16[~nan16])


def test_out_of_range_ids(rt, ctx, g4):
    g = golden("ple_w4_golden.npz")
    tab = rt.PleW4Table(ctx, g["packed"], g["scales"])
    with pytest.raises(g4.G4Error, match="PLE token id out of range: 24"):
        tab.rows_to_gpu(np.array([0, 24], np.int32))
    with pytest.raises(g4.G4Error, match="out of range"):
        tab.rows_to_gpu(np.array([-1], np.int32))
    # device ids: the kernel writes zero rows and raises the device error word
    out = tab.rows_to_gpu(torch.tensor([1, 99], dtype=torch.int32, device="cuda"), torch.float32)
    with pytest.raises(g4.G4Error, match="out-of-range"):
        ctx.check_device()
    assert float(out[1].abs().sum()) == 0.0
    ctx.check_device()  # cleared


def test_empty_batch(rt, ctx):
    g = golden("ple_w4_golden.npz")
    tab = rt.PleW4Table(ctx, g["packed"], g["scales"])
    assert tab.rows_to_gpu(np.zeros(0, np.int32)).shape == (0, 8960)


def test_streamed_shard_upload(rt, ctx, oracle):
    g = golden("ple_w4_golden.npz")
    tab = rt.PleW4Table(ctx, None, None, vocab=24, width=8960)
    for r0 in range(0, 24, 8):  # one "shard" at a time, as the reference streams them
        tab.upload_rows(r0, g["packed"][r0:r0 + 8], g["scales"][r0:r0 + 8])
    ids = np.arange(24, dtype=np.int32)
    assert np.array_equal(_bits(tab.rows_to_gpu(ids, torch.bfloat16)), g["expected_bf16"].view(np.int16))


def test_full_size_config2_properties(rt, ctx, oracle):
    """benchmark config 2 at full size: [262144, 8960] table, 4096 ids; sampled rows are
    bit-exact against the oracle and every output row sums to its table row's value."""
    vocab, width, T = 262144, 8960, 4096
    gen = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randint(-7, 8, (vocab, width // 2, 2), device="cuda", dtype=torch.int16, generator=gen)
    nib = (q & 0xF).to(torch.uint8)
    packed = (nib[..., 0] | (nib[..., 1] << 4)).contiguous()
    del q, nib
    sc = torch.randn((vocab, width // 32), device="cuda", generator=gen).abs_().mul_(0.05).to(torch.bfloat16)
    tab = rt.PleW4Table(ctx, packed, sc)
    ids = torch.randint(0, vocab, (T,), device="cuda", dtype=torch.int32, generator=gen)
    out = tab.rows_to_gpu(ids, torch.bfloat16)
    ctx.check_device()
    sample = torch.arange(0, T, 61, device="cuda")
    rows = ids[sample].long()
    p_h = packed[rows].cpu().numpy()
    s_h = sc[rows].view(torch.int16).cpu().numpy().view(np.uint16)
    ref = oracle.ple_read_rows(p_h, s_h, np.arange(len(sample), dtype=np.int32), bf16=True)
    assert np.array_equal(_bits(out[sample]).view(np.uint16), ref)
    again = tab.rows_to_gpu(ids, torch.bfloat16)
    assert torch.equal(out, again)
    del tab, packed, sc
    torch.cuda.empty_cache()


@pytest.mark.parametrize("width", [256, 512, 9216])
def test_other_widths_bit_exact(rt, ctx, oracle, width):
    """Widths other than the table's 8960 columns take the generic kernel instance: 16-byte
    scale loads when the groups fill whole vectors (512, 9216), scalar ones otherwise (256),
    and more words per row than one pass of the CTA (9216); f32 and bf16 bit-exact."""
    rng = np.random.default_rng(width)
    vocab = 50
    q = rng.integers(-7, 8, size=(vocab, width), dtype=np.int8)
    nib = (q.astype(np.int16) & 0xF).astype(np.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    scales = oracle.f32_to_bf16_bits(np.abs(rng.normal(0, 0.05, (vocab, width // 32))).astype(np.float32))
    tab = rt.PleW4Table(ctx, packed, scales, width=width)
    ids = rng.integers(0, vocab, 77).astype(np.int32)
    for dt, bf in ((torch.float32, False), (torch.bfloat16, True)):
        out = tab.rows_to_gpu(ids, dt)
        ref = oracle.ple_read_rows(packed, scales, ids, bf16=bf)
        assert np.array_equal(_bits(out), ref.view(np.int32 if not bf else np.int16))
    ctx.check_device()
