"""The oracle against golden vectors produced by the reference's own ``ref``
package (tests/golden/make_golden.py).  CPU only.

Pins: 16-bit outputs equal the reference bit for bit except for a few
outputs one unit in the last place away (summation order of the GEMM, last-bit
differences of exp, where the scaled GEMM applies its scales); fp32 outputs
within 1e-6 of max|ref|.  The scaled-GEMM goldens come from the reference
tests' own oracle (tests/gemm/test_triton.py:104-107), and the fp8 codec is
pinned to torch's float8 conversions.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from cases import all_cases, make_inputs, oracle_output, sampled
from oracle import ops

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = all_cases()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "golden.npz")


@pytest.fixture(scope="module")
def manifest():
    return json.loads((GOLDEN / "manifest.json").read_text())


def _from_bits(b: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return ops.bf16_from_bits(b)
    if dtype == "float16":
        return b.view(np.float16).astype(np.float32)
    return b.view(np.float32)


def _bits(x: np.ndarray, dtype: str) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "bfloat16":
        return ops.bf16_bits(x)
    if dtype == "float16":
        return x.astype(np.float16).view(np.uint16)
    return x.view(np.uint32)


def _ulp(x: np.ndarray, dtype: str) -> np.ndarray:
    mant = {"bfloat16": 7, "float16": 10, "float32": 23}[dtype]
    tiny = {"bfloat16": 2.0**-133, "float16": 2.0**-24, "float32": 2.0**-149}[dtype]
    e = np.floor(np.log2(np.maximum(np.abs(x), 1e-38)))
    return np.maximum(2.0 ** (e - mant), tiny)


def test_golden_covers_every_case(golden, manifest):
    assert set(golden.files) == {c.id for c in CASES}
    assert set(manifest["cases"]) == {c.id for c in CASES}


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.id)
def test_inputs_regenerate_bit_exact(case, manifest):
    def digest(x):
        raw = np.ascontiguousarray(x) if case.op == "scaled_gemm" else _bits(x, case.dtype)
        return hashlib.sha256(raw.tobytes()).hexdigest()

    digests = [digest(x) for x in make_inputs(case)]
    assert digests == manifest["cases"][case.id]["input_sha256"]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.id)
def test_oracle_matches_reference(case, golden):
    out = sampled(case, oracle_output(case, make_inputs(case)))
    ref = _from_bits(golden[case.id], case.dtype).reshape(out.shape)
    both_nan = np.isnan(out) & np.isnan(ref)
    diff = np.where(both_nan, 0.0, np.abs(out.astype(np.float64) - ref.astype(np.float64)))
    if case.dtype == "float32":
        scale = float(np.max(np.abs(ref))) or 1.0
        assert float(diff.max()) <= 1e-6 * scale
    else:
        bound = _ulp(ref, case.dtype)
        if case.op == "gemm":
            # fp32 accumulation in a different order: the two sums differ by up
            # to K * 2^-24 * sum_k |a_ik b_kj| before the final rounding.
            a, b = make_inputs(case)
            mag = sampled(case, np.abs(a) @ np.abs(b))
            bound = bound + case.shape[1] * 2.0**-24 * mag
        if case.op == "scaled_gemm":
            # The reference scales the operands before an fp32 matmul, the
            # oracle scales the accumulator: both round each scaled operand or
            # product and the fp32 sum, K + 2 roundings of 2^-24 at most.
            a_q, b_q, sa, sb = make_inputs(case)
            a = np.abs(ops.dequant(a_q, case.qdtype)) * np.abs(sa.reshape(-1, 1))
            b = np.abs(ops.dequant(b_q, case.qdtype)) * np.abs(sb.reshape(1, -1))
            bound = bound + (case.shape[1] + 2) * 2.0**-24 * (a @ b)
        assert np.all(diff <= bound), "a 16-bit output is more than one ulp off"
        assert np.mean(diff == 0) >= (0.99 if case.op == "scaled_gemm" else 0.999)


@pytest.mark.parametrize("kind", ["e4m3", "e5m2"])
def test_fp8_codec_matches_torch(kind):
    """fp8_encode / fp8_decode against torch's CPU float8 conversions (the
    conversion the reference's tests quantise with), over all 256 codes and
    1.2M values spanning subnormals, rounding ties and overflow."""
    torch = pytest.importorskip("torch")
    tdt = {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2}[kind]
    codes = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(codes).view(tdt).float().numpy()
    assert np.array_equal(ops.fp8_decode(codes, kind), want, equal_nan=True)
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(150_000).astype(np.float32) * np.float32(s)
                        for s in (1e-4, 1e-2, 1.0, 10.0, 1e2, 1e3, 1e4, 1e5)])
    # midpoints between neighbouring codes (ties) and the overflow edges
    vals = ops.fp8_decode(codes[:127], kind).astype(np.float64)
    vals = vals[np.isfinite(vals)]
    mids = ((vals[1:] + vals[:-1]) / 2).astype(np.float32)
    edges = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 464, 465, 480, 59392, 59391, 61440],
                     dtype=np.float32)
    x = np.concatenate([x, mids, -mids, edges])
    want = torch.from_numpy(x).to(tdt).view(torch.uint8).numpy()
    assert np.array_equal(ops.fp8_encode(x, kind), want)


def test_scaled_gemm_int8_is_exact():
    """int8 products summed in float64 are exact; the scaled result equals an
    integer matmul scaled in fp32."""
    from oracle.inputs import quantized, scales

    a = quantized((33, 70), 1, "int8")
    b = quantized((70, 17), 2, "int8")
    sa, sb = scales(33, 17, "row", 3)
    acc = (a.astype(np.int64) @ b.astype(np.int64)).astype(np.float32)
    want = ops.round_to((acc * sa.reshape(-1, 1)) * sb.reshape(1, -1), "float32")
    assert np.array_equal(ops.scaled_gemm(a, b, sa, sb, "int8", "float32"), want)


def test_special_values():
    x = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e30, -1e30, 88.0, -88.0, 1e-30],
                 dtype=np.float32)
    s = ops.silu(x, "float32")
    assert s[0] == 0 and s[2] == np.inf and np.isnan(s[4]) and s[5] == np.float32(1e30)
    assert s[6] == 0 and np.isnan(s[3])  # -inf / (1 + inf) is NaN, as in torch
    r = ops.relu(x, "float32")
    assert r[3] == 0 and np.isnan(r[4]) and r[2] == np.inf


def test_rounding_is_round_to_nearest_even():
    x = np.array([1.0 + 2.0**-8, 1.0 + 3 * 2.0**-8, 65536.0 * 2.0**-1], dtype=np.float32)
    assert list(ops.bf16_bits(x)) == [0x3F80, 0x3F82, 0x4700]
    assert ops.round_to(np.float32(70000.0), "float16") == np.inf


def test_sharded_block_matches_unsharded_block():
    from oracle.inputs import randn

    T, H, inter = 16, 64, 96
    x = randn((T, H), 1)
    nw = randn((H,), 2, mean=1.0, std=0.1)
    wgu = randn((H, 2 * inter), 3, std=0.02 * 8)
    wd = randn((inter, H), 4, std=0.02 * 8)
    full = ops.mlp_block(x, nw, wgu, wd, 1e-6, "bfloat16")
    for world in (1, 2, 4):
        part = ops.mlp_block_sharded(x, nw, wgu, wd, 1e-6, "bfloat16", world)
        err = np.max(np.abs(part - full))
        assert err <= 2e-2 * np.max(np.abs(full))


def test_folded_norm_oracle_tracks_the_reference_composition():
    """gemm_silu_mul_folded (rms_norm folded into the weight rows and the
    accumulator) against the reference composition ref.rmsnorm -> ref.gemm
    -> ref.silu(gate) * up restated by the pinned primitives: within the
    GEMM tolerance, and rms_rstd is the factor rmsnorm applies."""
    from oracle.inputs import randn

    x = randn((64, 512), 11)
    nw = randn((512,), 12, mean=1.0, std=0.1)
    wg = randn((512, 256), 13, std=512 ** -0.5)
    wu = randn((512, 256), 14, std=512 ** -0.5)
    folded = ops.gemm_silu_mul_folded(x, nw, wg, wu, 1e-6, "bfloat16")
    h = ops.rmsnorm(x, nw, 1e-6, "bfloat16")
    composed = ops.silu_mul_composed(ops.gemm(h, wg, "bfloat16"), ops.gemm(h, wu, "bfloat16"),
                                     "bfloat16")
    assert np.abs(folded - composed).max() <= 2e-2 * np.abs(composed).max()
    rstd = ops.rms_rstd(x, 1e-6)
    unit = ops.rmsnorm(x, np.ones(512, np.float32), 1e-6, "float32")
    np.testing.assert_allclose(unit, x * rstd.reshape(-1, 1), rtol=1e-6, atol=0)
