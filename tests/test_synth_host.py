"""Host side of the synthetic tensor generator (CPU only): determinism, the
normal variates, and that every block encoder writes blocks which an
independent decoder (gguf-py) reads back close to the generated values."""
import numpy as np
import pytest

from qmoe import synth
from qmoe.quant import GgmlType, calculate_tensor_bytes


def _gen(ty, n, seed=7, sid=3, sigma=1.0):
    b = np.empty(calculate_tensor_bytes(ty, n), dtype=np.uint8)
    synth.fill(b, ty, n, seed, sid, sigma)
    return b


def test_deterministic_and_seeded():
    a = _gen(GgmlType.Q4_K, 4096)
    b = _gen(GgmlType.Q4_K, 4096)
    c = _gen(GgmlType.Q4_K, 4096, seed=8)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)


def test_normal_moments():
    x = _gen(GgmlType.F32, 1 << 18).view(np.float32)
    assert abs(float(x.mean())) < 0.01
    assert abs(float(x.std()) - 1.0) < 0.01
    assert float(np.abs(x).max()) <= 6.0


@pytest.mark.parametrize("ty,tol", [(GgmlType.Q8_0, 0.006), (GgmlType.Q4_0, 0.08), (GgmlType.Q5_0, 0.04),
                                    (GgmlType.Q4_K, 0.08), (GgmlType.Q5_K, 0.04), (GgmlType.Q6_K, 0.02),
                                    (GgmlType.F16, 1e-3), (GgmlType.BF16, 8e-3)])
def test_encoder_roundtrip_via_gguf(ty, tol):
    from gguf import GGMLQuantizationType, quants
    n = 8192
    ref = _gen(GgmlType.F32, n).view(np.float32)   # the values the encoder saw
    raw = _gen(ty, n)
    dec = quants.dequantize(raw, GGMLQuantizationType(int(ty))).astype(np.float32).ravel()
    # error relative to the block's largest magnitude
    be = 256 if ty in (GgmlType.Q4_K, GgmlType.Q5_K, GgmlType.Q6_K) else 32
    amax = np.repeat(np.abs(ref).reshape(-1, be).max(axis=1), be)
    rel = np.abs(dec - ref) / np.maximum(amax, 1e-6)
    assert float(rel.max()) < tol, float(rel.max())


def test_oracle_reads_encoders_like_gguf():
    from gguf import GGMLQuantizationType, quants
    from oracle import oracle as orc
    for ty in (GgmlType.Q8_0, GgmlType.Q4_K, GgmlType.Q5_K, GgmlType.Q6_K, GgmlType.Q4_0, GgmlType.Q5_0):
        n = 2048
        raw = _gen(ty, n, sigma=0.02)
        dec = quants.dequantize(raw, GGMLQuantizationType(int(ty))).astype(np.float32).ravel()
        got = orc.dequant_row(raw, int(ty), n, 0, n)
        assert np.max(np.abs(got - dec)) <= 1e-7, ty
