"""Pin the CPU oracle against golden vectors produced by the reference's own
torch path (tests/golden/make_golden.py)."""

import hashlib

import numpy as np
import pytest
import torch

import oracle
from cdl_b200 import workloads

FMTS = {"nvfp4": oracle.NVFP4, "mxfp4": oracle.MXFP4, "mxfp8": oracle.MXFP8}


def _cases(golden):
    keys = sorted({k.rsplit("/", 1)[0] for k in golden.files if not k.startswith("swizzle/")})
    return keys


def test_golden_has_all_formats(golden):
    keys = _cases(golden)
    for name in FMTS:
        assert any(k.startswith(name + "/") for k in keys)
    assert len(keys) >= 20


def test_oracle_quant_matches_reference(golden):
    for key in _cases(golden):
        fmt = FMTS[key.split("/")[0]]
        x = golden[key + "/x"]
        packed, scale, alpha = oracle.quant(x, fmt)
        np.testing.assert_array_equal(packed, golden[key + "/packed"], err_msg=key)
        np.testing.assert_array_equal(scale, golden[key + "/scale"], err_msg=key)
        if fmt == oracle.NVFP4:
            assert alpha.view(np.uint32)[0] == golden[key + "/alpha"].view(np.uint32)[0], key


def test_wide_oracle_matches_reference_on_bf16_values(golden):
    """The fp32 / fp16 oracle (the Triton kernel's fp32 arithmetic) on the
    golden inputs widened to fp32 gives the reference's golden codes, scales
    and alpha; on fp16-representable values its fp16 and fp32 inputs agree."""
    from oracle.wide import quant_wide

    for key in _cases(golden):
        fmt = FMTS[key.split("/")[0]]
        x = oracle.bf16_bits_to_f32(golden[key + "/x"])
        packed, scale, alpha = quant_wide(x, fmt)
        np.testing.assert_array_equal(packed, golden[key + "/packed"], err_msg=key)
        np.testing.assert_array_equal(scale, golden[key + "/scale"], err_msg=key)
        if fmt == oracle.NVFP4:
            assert alpha.view(np.uint32)[0] == golden[key + "/alpha"].view(np.uint32)[0], key
    rng = np.random.default_rng(3)
    h = (rng.standard_normal((64, 96)) * np.exp(rng.standard_normal((64, 1)))).astype(np.float16)
    for fmt in FMTS.values():
        for a, b in zip(quant_wide(h, fmt), quant_wide(h.astype(np.float32), fmt)):
            if a is not None:
                np.testing.assert_array_equal(a, b)


def test_oracle_dequant_matches_reference(golden):
    for key in _cases(golden):
        fmt = FMTS[key.split("/")[0]]
        alpha = golden[key + "/alpha"] if fmt == oracle.NVFP4 else (np.ones(1, np.float32) if fmt == oracle.MXFP4 else None)
        deq = oracle.dequant(golden[key + "/packed"], golden[key + "/scale"], fmt, alpha)
        np.testing.assert_array_equal(deq, golden[key + "/deq"], err_msg=key)


def test_oracle_swizzle_matches_reference(golden):
    for key in sorted({k.rsplit("/", 1)[0] for k in golden.files if k.startswith("swizzle/")}):
        np.testing.assert_array_equal(oracle.swizzle(golden[key + "/in"]), golden[key + "/out"], err_msg=key)


def test_e4m3_roundtrip_all_bytes():
    vals = oracle.e4m3_values(np.arange(256, dtype=np.uint8))
    for b in range(256):
        if (b & 0x7F) == 0x7F:
            continue
        assert oracle._load().oracle_f32_to_e4m3(float(vals[b])) == b
    ref = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    fin = np.isfinite(ref)
    np.testing.assert_array_equal(vals[fin], ref[fin])


def test_e4m3_rounding_matches_torch():
    g = torch.Generator().manual_seed(5)
    v = torch.cat([
        (torch.rand(200000, generator=g) * 2 - 1) * 448,
        (torch.rand(100000, generator=g) * 2 - 1) * 2.0**-6,
        torch.tensor([2.0**-10, 3 * 2.0**-10, 2.0**-10 * 1.0000001, 0.0, -0.0, 448.0, -448.0]),
    ])
    ref = v.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    lib = oracle._load()
    got = np.array([lib.oracle_f32_to_e4m3(float(f)) for f in v.numpy()], np.uint8)
    np.testing.assert_array_equal(got, ref)


def _bits(x):
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_oracle_c1_digest(digests):
    d = digests["c1_nvfp4_4096x4096"]
    x = _bits(workloads.c1_nvfp4())
    assert _sha(x) == d["input"]
    packed, scale, alpha = oracle.quant(x, oracle.NVFP4)
    assert _sha(packed) == d["packed"]
    assert _sha(scale) == d["scale"]
    assert int(alpha.view(np.int32)[0]) == d["alpha_bits"]
    assert _sha(oracle.dequant(packed, scale, oracle.NVFP4, alpha)) == d["deq"]


@pytest.mark.parametrize("k", [2048, 8192])
def test_oracle_c2_digests(digests, k):
    x = workloads.c2_mx(16384, k, seed=0)
    for tag, inp in (("rows", x), ("transposed", x.t().contiguous())):
        xb = _bits(inp)
        for name, fmt in (("mxfp4", oracle.MXFP4), ("mxfp8", oracle.MXFP8)):
            d = digests[f"c2_{name}_16384x{k}_{tag}"]
            assert _sha(xb) == d["input"]
            packed, scale, alpha = oracle.quant(xb, fmt)
            assert _sha(packed) == d["packed"], (name, k, tag)
            assert _sha(scale) == d["scale"], (name, k, tag)
            assert _sha(oracle.dequant(packed, scale, fmt, alpha)) == d["deq"], (name, k, tag)
