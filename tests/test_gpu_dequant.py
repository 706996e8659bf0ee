"""Load-time dequantisation on the GPU, bit for bit against the CPU
restatement of quant.rs (and, for the f32->f16 step, against the reference's
integer rounding over every f32 bit pattern)."""
import numpy as np
import pytest

import hotseat_b200 as hs
from oracle import ffi

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

BLOCKS = {12: (144, 256), 14: (210, 256), 8: (34, 32), 6: (22, 32), 13: (176, 256), 1: (2, 1), 0: (4, 1)}
F16_OFFSETS = {12: (0, 2), 13: (0, 2), 14: (208,), 8: (0,), 6: (0,)}


def random_blocks(ty, nb, rng):
    bs, be = BLOCKS[ty]
    if ty == 1:
        return (rng.standard_normal(nb) * 3).astype(np.float16).view(np.uint8).reshape(nb, 2)
    if ty == 0:
        return (rng.standard_normal(nb) * 10.0 ** rng.uniform(-9, 5, nb)).astype(np.float32).view(np.uint8).reshape(nb, 4)
    r = rng.integers(0, 256, size=(nb, bs), dtype=np.uint8)
    for off in F16_OFFSETS[ty]:
        r[:, off:off + 2] = (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return r


def device_dequant(ty, raw, n, src_offset=0):
    src = torch.zeros(raw.size + 16, dtype=torch.uint8, device="cuda")
    src[src_offset:src_offset + raw.size] = torch.from_numpy(raw.reshape(-1)).cuda()
    dst = torch.zeros(n, dtype=torch.int16, device="cuda")
    hs.dequant_f16(ty, src.data_ptr() + src_offset, n, dst.data_ptr())
    torch.cuda.synchronize()
    return dst.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("ty", sorted(BLOCKS))
@pytest.mark.parametrize("nb", [1, 7, 1000, 50_001])
def test_dequant_random_blocks_bit_exact(ty, nb):
    rng = np.random.default_rng(ty * 1000 + nb)
    raw = random_blocks(ty, nb, rng)
    n = nb * BLOCKS[ty][1]
    assert np.array_equal(device_dequant(ty, raw, n), ffi.dequant_f16(ty, raw.tobytes(), n))


@pytest.mark.parametrize("ty", [12, 14])
def test_dequant_unaligned_source_takes_the_scalar_path(ty):
    rng = np.random.default_rng(1)
    raw = random_blocks(ty, 333, rng)
    n = 333 * 256
    assert np.array_equal(device_dequant(ty, raw, n, src_offset=3), ffi.dequant_f16(ty, raw.tobytes(), n))


def test_f32_to_f16_matches_the_reference_rounding_for_every_f32():
    """f16.rs:35-69 restated in integer torch ops on the GPU, compared with the
    kernel's conversion for all 2^32 f32 bit patterns (NaNs only need to stay NaN)."""
    chunk = 1 << 27
    for c in range(32):
        bits = torch.arange(c * chunk, (c + 1) * chunk, dtype=torch.int64, device="cuda")
        src = bits.to(torch.int32)  # wraps to the same 32-bit patterns
        out = torch.empty(chunk, dtype=torch.int16, device="cuda")
        hs.dequant_f16(0, src.data_ptr(), chunk, out.data_ptr())
        x = bits
        sign = (x >> 16) & 0x8000
        exp = ((x >> 23) & 0xFF) - 112
        man = x & 0x7FFFFF
        is_nan = (((x >> 23) & 0xFF) == 0xFF) & (man != 0)
        # normal path
        half = (exp << 10) | (man >> 13)
        rem = man & 0x1FFF
        rnd = ((rem > 0x1000) | ((rem == 0x1000) & (((man >> 13) & 1) == 1))).to(torch.int64)
        normal = (half + rnd) | sign
        # subnormal path
        m = man | 0x800000
        shift = (14 - exp).clamp(min=1, max=31)
        h2 = m >> shift
        rem2 = m & ((torch.ones_like(shift) << shift) - 1)
        tie = torch.ones_like(shift) << (shift - 1)
        rnd2 = ((rem2 > tie) | ((rem2 == tie) & ((h2 & 1) == 1))).to(torch.int64)
        sub = sign | (h2 + rnd2)
        want = torch.where(exp >= 0x1F, sign | 0x7C00, torch.where(exp <= 0, torch.where(exp < -10, sign, sub), normal))
        inf = ((x >> 23) & 0xFF) == 0xFF
        want = torch.where(inf & ~is_nan, sign | 0x7C00, want)
        got = out.to(torch.int64) & 0xFFFF
        bad = (got != want) & ~is_nan
        assert int(bad.sum()) == 0, f"chunk {c}: {int(bad.sum())} mismatches"
        nan_ok = ((got & 0x7C00) == 0x7C00) & ((got & 0x3FF) != 0)
        assert bool(nan_ok[is_nan].all())


def test_model_tensors_bit_exact_on_the_05b_shape(q05_gguf):
    m = hs.Model.load(q05_gguf, max_ctx=64)
    o = ffi.Model(q05_gguf, max_ctx=64)
    assert m.fingerprint == o.cfg.fingerprint
    for name in ["token_embd.weight", "blk.0.ffn_gate.weight", "blk.0.ffn_down.weight", "blk.23.ffn_up.weight",
                 "blk.5.attn_k.weight", "blk.11.attn_q.weight", "blk.17.attn_output.weight"]:
        assert np.array_equal(m.tensor(name), o.tensor_f16(name)), name
    for name in ["blk.3.attn_q.bias", "blk.3.attn_norm.weight", "output_norm.weight"]:
        assert np.array_equal(m.tensor(name), o.tensor_f32(name)), name
