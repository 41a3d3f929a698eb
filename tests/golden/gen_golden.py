"""Generates tests/golden/quant_kat.json: the known-answer fixtures of the
reference's own kernel tests (sahan974/qwen-3.5-cuda tests/kernel_tests.cu).

  * quant blocks: tests/kernel_tests.cu:116-223 -- one hand-built block per
    type (Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K) with deliberately varied packed
    fields; the byte patterns below restate those fixture definitions.
    Expected values are computed twice, independently: with gguf-py's numpy
    decoders (gguf 0.19.0, an installed third-party implementation of the
    GGML layouts) and with the reference test's own expected-value equations
    (kernel_tests.cu:125-221, restated); the script asserts they agree.
  * routing: tests/kernel_tests.cu:424-453 -- logits, K and the expected ids.

Run:  python tests/golden/gen_golden.py    (needs numpy + gguf; no GPU)
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "quant_kat.json"

PACKED_SCALES = [0xC1, 0x82, 0x43, 0x04, 0x85, 0x46, 0x07, 0xC8, 0x91, 0x2A, 0xB3, 0x4C]  # kernel_tests.cu:159


def half_one(b: bytearray, off: int) -> None:  # kernel_tests.cu:37-40
    b[off], b[off + 1] = 0x00, 0x3C


def scale_min_ref(j: int, s) -> tuple[int, int]:  # kernel_tests.cu:106-114
    if j < 4:
        return s[j] & 63, s[j + 4] & 63
    return (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4), (s[j + 4] >> 4) | ((s[j] >> 6) << 4)


def fixtures():
    fx = {}
    # Q4_0 (:121-130)
    q = bytearray(18); half_one(q, 0)
    for j in range(16):
        q[2 + j] = (((15 - j) & 15) << 4 | (j & 15)) & 0xFF
    r = [0.0] * 32
    for j in range(16):
        r[j] = (q[2 + j] & 15) - 8
        r[j + 16] = (q[2 + j] >> 4) - 8
    fx["Q4_0"] = (2, bytes(q), r)
    # Q5_0 (:133-146)
    q = bytearray(22); half_one(q, 0)
    q[2], q[3], q[4], q[5] = 0x69, 0x96, 0x3C, 0xC3
    for j in range(16):
        q[6 + j] = (((j * 5 + 3) & 15) << 4 | ((j * 7 + 1) & 15)) & 0xFF
    qh = q[2] | (q[3] << 8) | (q[4] << 16) | (q[5] << 24)
    r = [0.0] * 32
    for j in range(16):
        r[j] = ((q[6 + j] & 15) | (((qh >> j) & 1) << 4)) - 16
        r[j + 16] = ((q[6 + j] >> 4) | (((qh >> (j + 16)) & 1) << 4)) - 16
    fx["Q5_0"] = (6, bytes(q), r)
    # Q8_0 (:149-157)
    q = bytearray(34); half_one(q, 0)
    r = [0.0] * 32
    for j in range(32):
        v = np.int8(np.int32(j * 7 - 101).astype(np.int8))
        q[2 + j] = int(v) & 0xFF
        r[j] = float(v)
    fx["Q8_0"] = (8, bytes(q), r)
    # Q4_K (:162-177)
    q = bytearray(144); half_one(q, 0)
    q[2], q[3] = 0x00, 0x38
    q[4:16] = bytes(PACKED_SCALES)
    for j in range(128):
        q[16 + j] = (((j * 11 + 5) & 15) << 4 | ((j * 3 + 1) & 15)) & 0xFF
    r = [0.0] * 256
    for i in range(256):
        sc, mn = scale_min_ref(i // 32, q[4:16])
        g, l = i // 64, i % 32
        b = q[16 + g * 32 + l]
        v = (b & 15) if (i % 64) < 32 else (b >> 4)
        r[i] = float(np.float32(sc * v) - np.float32(0.5) * np.float32(mn))
    fx["Q4_K"] = (12, bytes(q), r)
    # Q5_K (:180-197)
    q = bytearray(176); half_one(q, 0)
    q[2], q[3] = 0x00, 0x38
    q[4:16] = bytes(PACKED_SCALES)
    for j in range(32):
        q[16 + j] = (j * 37 + 13) & 0xFF
    for j in range(128):
        q[48 + j] = (((j * 9 + 2) & 15) << 4 | ((j * 5 + 7) & 15)) & 0xFF
    r = [0.0] * 256
    for i in range(256):
        sc, mn = scale_min_ref(i // 32, q[4:16])
        g, l = i // 64, i % 32
        b = q[48 + g * 32 + l]
        mask = 1 << (2 * g + (1 if (i % 64) >= 32 else 0))
        v = ((b & 15) if (i % 64) < 32 else (b >> 4)) + (16 if (q[16 + l] & mask) else 0)
        r[i] = float(np.float32(sc * v) - np.float32(0.5) * np.float32(mn))
    fx["Q5_K"] = (13, bytes(q), r)
    # Q6_K (:200-222)
    q = bytearray(210)
    for j in range(128):
        q[j] = (j * 29 + 7) & 0xFF
    for j in range(64):
        q[128 + j] = (j * 43 + 19) & 0xFF
    for j in range(16):
        q[192 + j] = (j * 9 - 61) & 0xFF
    half_one(q, 208)
    r = [0.0] * 256
    for i in range(256):
        half, rr = i // 128, i % 128
        lane, quarter = rr & 31, rr // 32
        lo = [q[half * 64 + lane] & 15, q[half * 64 + 32 + lane] & 15, q[half * 64 + lane] >> 4,
              q[half * 64 + 32 + lane] >> 4][quarter]
        hi = (q[128 + half * 32 + lane] >> (2 * quarter)) & 3
        si = half * 8 + lane // 16 + 2 * quarter
        scale = q[192 + si] - 256 if q[192 + si] >= 128 else q[192 + si]
        r[i] = float(scale * ((lo | (hi << 4)) - 32))
    fx["Q6_K"] = (14, bytes(q), r)
    return fx


def gguf_decode(name: str, raw: bytes) -> np.ndarray:
    from gguf import GGMLQuantizationType, quants
    t = getattr(GGMLQuantizationType, name)
    return quants.dequantize(np.frombuffer(raw, dtype=np.uint8), t).astype(np.float32).ravel()


def main() -> None:
    out = {"source": "tests/kernel_tests.cu:116-223 and :424-453 of sahan974/qwen-3.5-cuda", "quant": {}}
    for name, (tid, raw, expect) in fixtures().items():
        ind = gguf_decode(name, raw)
        exp = np.array(expect, dtype=np.float32)
        err = float(np.max(np.abs(ind - exp)))
        assert err < 1e-6, (name, err)
        out["quant"][name] = {"ggml_type": tid, "bytes": raw.hex(), "expected": [float(v) for v in ind]}
    out["routing"] = {"logits": [-2.0, 0.4, 3.0, 1.2, -0.7, 2.1], "k": 3, "ids": [2, 5, 3],
                      "sum_tol": 1e-6, "abs_tol_quant": 1e-6}
    OUT.write_text(json.dumps(out, indent=1))
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
