"""Generate tests/golden/golden.json: known-answer vectors for the oracle and the CUDA path.

Two sources, both independent of oracle/oracle.c:

1. The reference's own known-answer tests, restated as data (each case cites
   the llmtoy-zig test it comes from).
2. Single-superblock Q4_K / Q6_K / Q8_0 vectors decoded here (every step
   exact in double, then one rounding to f32) from the block layouts documented in
   src/quant/dequant.zig:31-40,136-155,219-235 (the reference has no
   non-zero Q4_K or any Q6_K known-answer test).  Each value is the f32 the
   reference's strict-float arithmetic produces: Q4_K's d1*q - m1 is one
   rounding of an exact quantity (d1*q and m1 are exact in f32), Q6_K's and
   Q8_0's products are exact.  The same for Q5_0, Q5_1, Q5_K, Q3_K and IQ4_NL
   (dequant.zig:196-217,307-506,615-640): Q5_1's d*q + m and Q5_K's d1*q - m1
   are rounded once from the exact rational value; the other products are
   exact.  Q8_1 activation blocks (dequant.zig:508-613) are quantised here with
   numpy float32 arithmetic (IEEE-rounded division and products, halves
   rounded away from zero as Zig's @round does, f16 by round-to-nearest-even).

Run:  python tests/golden/gen_golden.py   (deterministic; rewrites golden.json)
"""
from __future__ import annotations

import json
import math
import struct
from fractions import Fraction
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().with_name("golden.json")


def f16_value(bits: int) -> Fraction:
    sign = -1 if bits & 0x8000 else 1
    exp = (bits >> 10) & 0x1F
    mant = bits & 0x3FF
    if exp == 0:
        return sign * Fraction(mant, 1 << 24)
    if exp == 31:
        raise ValueError("inf/nan not used in fixtures")
    return sign * Fraction(1024 + mant, 1024) * (Fraction(2) ** (exp - 15))


def f32_bits(v: float) -> int:
    """Round a double to f32 (nearest-even) and return its bit pattern.

    Every value passed here was computed exactly in double (products of at
    most 24-bit operands, one difference), so this is the single rounding the
    reference's f32 arithmetic performs, signed zeros included."""
    return struct.unpack("<I", struct.pack("<f", v))[0]


def bits_to_f32(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b))[0]


# ── independent block decoders (exact) ────────────────────────────────────────

def q8_0_decode(blk: bytes) -> list[int]:
    d = float(f16_value(blk[0] | blk[1] << 8))
    out = []
    for i in range(32):
        q = blk[2 + i] - 256 if blk[2 + i] >= 128 else blk[2 + i]
        out.append(f32_bits(d * float(q)))
    return out


def k4_scale_min(j: int, s: bytes) -> tuple[int, int]:
    if j < 4:
        return s[j] & 63, s[j + 4] & 63
    return (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4), (s[j + 4] >> 4) | ((s[j] >> 6) << 4)


def q4k_decode(blk: bytes) -> list[int]:
    d, dmin = float(f16_value(blk[0] | blk[1] << 8)), float(f16_value(blk[2] | blk[3] << 8))
    scales, qs = blk[4:16], blk[16:144]
    out = [0] * 256
    for e in range(256):
        c, p = divmod(e, 64)
        j = 2 * c + (1 if p >= 32 else 0)
        byte = qs[32 * c + (p & 31)]
        q = byte & 15 if p < 32 else byte >> 4
        sc, mn = k4_scale_min(j, scales)
        d1, m1 = d * float(sc), dmin * float(mn)  # exact: <= 17 significant bits
        out[e] = f32_bits(d1 * float(q) - m1)
    return out


def f32_round_exact(x: Fraction) -> int:
    """Bit pattern of the f32 nearest to the rational x (ties to even)."""
    if x == 0:
        return 0x80000000 if x < 0 else 0
    sign = 0x80000000 if x < 0 else 0
    a = abs(x)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    e = max(e, -126)
    m = a / Fraction(2) ** (e - 23)  # in [2^23, 2^24) for normals
    q, r = divmod(m.numerator, m.denominator)
    if 2 * r > m.denominator or (2 * r == m.denominator and q & 1):
        q += 1
    if q >= 1 << 24:
        q >>= 1
        e += 1
    if q < 1 << 23:  # subnormal
        return sign | q
    return sign | ((e + 127) << 23) | (q - (1 << 23))


def f32_of(exact: Fraction, approx: float) -> int:
    """One rounding of an exact sum; an exact zero takes its sign from the
    same sum in double, which follows IEEE's signed-zero rules."""
    return f32_bits(approx) if exact == 0 else f32_round_exact(exact)


def q5_bits(qh: int, qs: bytes) -> list[int]:
    """The 32 five-bit values: element j < 16 = low nibble of qs[j] | bit j of
    qh << 4, element j + 16 = high nibble | bit j + 16 << 4."""
    return [((qs[e] & 15) if e < 16 else (qs[e - 16] >> 4)) | (((qh >> e) & 1) << 4) for e in range(32)]


def q5_0_decode(blk: bytes) -> list[int]:
    d = f16_value(blk[0] | blk[1] << 8)
    qh = int.from_bytes(blk[2:6], "little")
    return [f32_bits(float(d) * (v - 16)) for v in q5_bits(qh, blk[6:22])]  # exact products


def q5_1_decode(blk: bytes) -> list[int]:
    d, m = f16_value(blk[0] | blk[1] << 8), f16_value(blk[2] | blk[3] << 8)
    qh = int.from_bytes(blk[4:8], "little")
    # d * q is exact in f32 (11 x 5 bits); the sum rounds once
    return [f32_of(d * v + m, float(d) * v + float(m)) for v in q5_bits(qh, blk[8:24])]


IQ4_TABLE = [-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113]


def iq4nl_decode(blk: bytes) -> list[int]:
    d = f16_value(blk[0] | blk[1] << 8)
    nib = [(blk[2 + e] & 15) if e < 16 else (blk[2 + e - 16] >> 4) for e in range(32)]
    return [f32_bits(float(d) * IQ4_TABLE[n]) for n in nib]


def q5k_decode(blk: bytes) -> list[int]:
    d, dmin = f16_value(blk[0] | blk[1] << 8), f16_value(blk[2] | blk[3] << 8)
    scales, qh, ql = blk[4:16], blk[16:48], blk[48:176]
    out = [0] * 256
    for e in range(256):
        c, p = divmod(e, 64)
        up = 1 if p >= 32 else 0
        byte = ql[32 * c + (p & 31)]
        q = (byte >> 4 if up else byte & 15) + 16 * ((qh[p & 31] >> (2 * c + up)) & 1)
        sc, mn = k4_scale_min(2 * c + up, scales)
        # d*sc, dmin*mn and d1*q are exact in f32; the difference rounds once
        out[e] = f32_of(d * sc * q - dmin * mn, float(d) * sc * q - float(dmin) * mn)
    return out


def q3k_scales(s: bytes) -> list[int]:
    """16 six-bit scales: low nibbles of bytes 0-7 then their high nibbles,
    each with two high bits from byte 8 + k % 4 at bit 2 * (k // 4)."""
    out = []
    for k in range(16):
        w, b = divmod(k, 4)
        byte = s[4 * (w & 1) + b]
        lo = byte >> 4 if w & 2 else byte & 15
        out.append(lo | (((s[8 + b] >> (2 * w)) & 3) << 4))
    return out


def q3k_decode(blk: bytes) -> list[int]:
    hmask, qs, sc = blk[0:32], blk[32:96], q3k_scales(blk[96:108])
    d = f16_value(blk[108] | blk[109] << 8)
    out = [0] * 256
    for e in range(256):
        h, r = divmod(e, 128)
        j, r2 = divmod(r, 32)
        g, l = divmod(r2, 16)
        lo2 = (qs[32 * h + 16 * g + l] >> (2 * j)) & 3
        hb = (hmask[16 * g + l] >> (4 * h + j)) & 1
        out[e] = f32_bits(float(lo2 - (0 if hb else 4)) * (float(d) * (sc[8 * h + 2 * j + g] - 32)))
    return out


def pack_q3k_scales(sc: list[int]) -> bytes:
    b = bytearray(12)
    for k, v in enumerate(sc):
        w, i = divmod(k, 4)
        if w & 2:
            b[4 * (w & 1) + i] |= (v & 15) << 4
        else:
            b[4 * (w & 1) + i] |= v & 15
        b[8 + i] |= ((v >> 4) & 3) << (2 * w)
    return bytes(b)


def q8_1_quantize(x: np.ndarray) -> bytes:
    """quantizeQ8_1 (dequant.zig:517-547) in numpy float32 arithmetic."""
    out = bytearray()
    for b in range(len(x) // 32):
        src = np.asarray(x[32 * b:32 * b + 32], dtype=np.float32)
        amax = np.float32(0)
        for v in src:
            if abs(v) > amax:
                amax = np.float32(abs(v))
        d = np.float32(amax / np.float32(127.0))
        inv = np.float32(np.float32(1.0) / d) if d != 0 else np.float32(0)
        qs = []
        for v in src:
            t = float(np.float32(v * inv))
            q = math.floor(abs(t) + 0.5) * (1 if t >= 0 else -1)
            qs.append(int(min(127, max(-127, q))))
        s = np.float32(d * np.float32(sum(qs)))
        out += np.float16(d).tobytes() + np.float16(s).tobytes() + bytes(q & 0xFF for q in qs)
    return bytes(out)


def q6k_decode(blk: bytes) -> list[int]:
    ql, qh, sc = blk[0:128], blk[128:192], blk[192:208]
    d = float(f16_value(blk[208] | blk[209] << 8))
    out = [0] * 256
    for e in range(256):
        n, r = divmod(e, 128)
        kind, l = divmod(r, 32)
        lo = (ql[64 * n + l + 32 * (kind & 1)] >> (4 * (kind >> 1))) & 15
        hi = (qh[32 * n + l] >> (2 * kind)) & 3
        s = sc[8 * n + l // 16 + 2 * kind]
        s = s - 256 if s >= 128 else s
        out[e] = f32_bits((d * float(s)) * float((lo | hi << 4) - 32))
    return out


def pack_k4_scales(sc: list[int], mn: list[int]) -> bytes:
    b = bytearray(12)
    for j in range(4):
        b[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6)
        b[j + 4] = (mn[j] & 63) | ((mn[j + 4] >> 4) << 6)
        b[j + 8] = (sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4)
    return bytes(b)


def h16(v: float) -> bytes:
    return np.array([v], dtype=np.float16).tobytes()


# ── fixtures ─────────────────────────────────────────────────────────────────

def dequant_cases() -> list[dict]:
    cases = []
    # dequant.zig:702-714 — Q8_0 d=0.5, q=[2,-2,4,0,...] -> [1,-1,2,0,...]
    blk = bytearray(34)
    blk[0], blk[1] = 0x00, 0x38
    blk[2], blk[3], blk[4] = 2, 0xFE, 4
    cases.append({"name": "q8_0_roundtrip (dequant.zig:702)", "type": 8, "cols": 32, "hex": blk.hex(),
                  "expect": q8_0_decode(bytes(blk))})
    # dequant.zig:760-766 — Q4_K all-zero block -> zeros
    cases.append({"name": "q4k_zero_block (dequant.zig:760)", "type": 12, "cols": 256, "hex": bytes(144).hex(),
                  "expect": [0] * 256})
    # dequant.zig:670-678 — F16 0x3C00 -> 1.0, 0xBC00 -> -1.0
    cases.append({"name": "f16 (dequant.zig:670)", "type": 1, "cols": 2, "hex": "003c00bc",
                  "expect": [f32_bits(1), f32_bits(-1)]})
    # hand-built Q4_K: every scale/min path incl. the split high bits (j >= 4)
    sc = [1, 2, 3, 63, 17, 33, 48, 62]
    mn = [0, 5, 63, 1, 16, 32, 47, 9]
    qs = bytes(((k * 7 + 3) & 0xFF) for k in range(128))
    blk = h16(0.5) + h16(0.25) + pack_k4_scales(sc, mn) + qs
    cases.append({"name": "q4k_hand_scales", "type": 12, "cols": 256, "hex": blk.hex(), "expect": q4k_decode(blk)})
    blk = h16(0.00213) + h16(0.00101) + pack_k4_scales([63] * 8, [63] * 8) + bytes([0xF0] * 128)
    cases.append({"name": "q4k_hand_extremes", "type": 12, "cols": 256, "hex": blk.hex(), "expect": q4k_decode(blk)})
    # subnormal f16 scale
    blk = bytes([0x01, 0x00, 0x03, 0x00]) + pack_k4_scales(sc, mn) + qs
    cases.append({"name": "q4k_subnormal_d", "type": 12, "cols": 256, "hex": blk.hex(), "expect": q4k_decode(blk)})
    # hand-built Q6_K: ql/qh patterns hitting every (kind, half) and signed scales
    ql = bytes(((k * 13 + 5) & 0xFF) for k in range(128))
    qh = bytes(((k * 29 + 11) & 0xFF) for k in range(64))
    scb = bytes(((s * 37 - 100) & 0xFF) for s in range(16))
    blk = ql + qh + scb + h16(0.0031)
    cases.append({"name": "q6k_hand", "type": 14, "cols": 256, "hex": blk.hex(), "expect": q6k_decode(blk)})
    blk = bytes([0xFF] * 128) + bytes([0xFF] * 64) + bytes([0x80, 0x7F] * 8) + h16(-0.75)
    cases.append({"name": "q6k_extremes", "type": 14, "cols": 256, "hex": blk.hex(), "expect": q6k_decode(blk)})
    # hand-built Q5_0 / Q5_1 / IQ4_NL blocks: every nibble and fifth-bit position
    qs = bytes(((j * 11 + 7) & 0xFF) for j in range(16))
    blk = h16(0.5) + (0xA5C3F00F).to_bytes(4, "little") + qs
    cases.append({"name": "q5_0_hand", "type": 6, "cols": 32, "hex": blk.hex(), "expect": q5_0_decode(blk)})
    blk = h16(-0.0625) + h16(3.0) + (0x5A3C0FF0).to_bytes(4, "little") + qs
    cases.append({"name": "q5_1_hand", "type": 7, "cols": 32, "hex": blk.hex(), "expect": q5_1_decode(blk)})
    blk = bytes([0x01, 0x00]) + h16(1e-7) + (0xFFFFFFFF).to_bytes(4, "little") + bytes([0xFF] * 16)
    cases.append({"name": "q5_1_subnormal_d", "type": 7, "cols": 32, "hex": blk.hex(), "expect": q5_1_decode(blk)})
    blk = h16(1.0) + bytes((i & 15) | ((15 - i) << 4) for i in range(16))
    cases.append({"name": "iq4_nl_table", "type": 20, "cols": 32, "hex": blk.hex(), "expect": iq4nl_decode(blk)})
    # hand-built Q5_K (Q4_K's scales, every qh bit plane) and Q3_K (all 16 scales incl. 0 and 63)
    blk = h16(0.5) + h16(0.25) + pack_k4_scales(sc, mn) + bytes(((k * 37 + 1) & 0xFF) for k in range(32)) + \
        bytes(((k * 7 + 3) & 0xFF) for k in range(128))
    cases.append({"name": "q5k_hand", "type": 13, "cols": 256, "hex": blk.hex(), "expect": q5k_decode(blk)})
    s3 = [0, 63, 32, 1, 31, 33, 17, 48, 5, 60, 40, 24, 12, 50, 2, 61]
    blk = bytes(((k * 53 + 9) & 0xFF) for k in range(32)) + bytes(((k * 91 + 4) & 0xFF) for k in range(64)) + \
        pack_q3k_scales(s3) + h16(0.01)
    assert q3k_scales(pack_q3k_scales(s3)) == s3
    cases.append({"name": "q3k_hand", "type": 11, "cols": 256, "hex": blk.hex(), "expect": q3k_decode(blk)})
    # seeded random superblocks, two per format, multi-block rows
    rng = np.random.Generator(np.random.PCG64(20261201))
    for t, nb, dec, nbytes, elems in ((12, 2, q4k_decode, 144, 256), (14, 2, q6k_decode, 210, 256),
                                      (8, 3, q8_0_decode, 34, 32)):
        raw = bytearray(rng.integers(0, 256, size=nb * nbytes, dtype=np.uint8).tobytes())
        for b in range(nb):  # keep f16 scales finite and small
            scale = h16(float(rng.uniform(1e-3, 4e-3)))
            if t == 14:
                raw[b * nbytes + 208:b * nbytes + 210] = scale
            else:
                raw[b * nbytes:b * nbytes + 2] = scale
                if t == 12:
                    raw[b * nbytes + 2:b * nbytes + 4] = h16(float(rng.uniform(0, 2e-3)))
        expect = []
        for b in range(nb):
            expect += dec(bytes(raw[b * nbytes:(b + 1) * nbytes]))
        cases.append({"name": f"random_type{t}", "type": t, "cols": nb * elems, "hex": bytes(raw).hex(),
                      "expect": expect})
    # the same for the further formats (a separate stream, so the cases above stay as they were)
    rng = np.random.Generator(np.random.PCG64(20261202))
    for t, nb, dec, nbytes, elems, scale_offs in ((6, 3, q5_0_decode, 22, 32, (0,)), (7, 3, q5_1_decode, 24, 32, (0, 2)),
                                                  (20, 3, iq4nl_decode, 18, 32, (0,)),
                                                  (13, 2, q5k_decode, 176, 256, (0, 2)),
                                                  (11, 2, q3k_decode, 110, 256, (108,))):
        raw = bytearray(rng.integers(0, 256, size=nb * nbytes, dtype=np.uint8).tobytes())
        for b in range(nb):
            for o in scale_offs:
                raw[b * nbytes + o:b * nbytes + o + 2] = h16(float(rng.uniform(-4e-3, 4e-3)))
        expect = []
        for b in range(nb):
            expect += dec(bytes(raw[b * nbytes:(b + 1) * nbytes]))
        cases.append({"name": f"random_type{t}", "type": t, "cols": nb * elems, "hex": bytes(raw).hex(),
                      "expect": expect})
    return cases


def dot_q5_0_case() -> dict:
    # dequant.zig:716-735: block 0 d=0.5, qh=0xAAAAAAAA, qs[j] = j | (j+3)<<4;
    # block 1 d=0.125, qh=0, qs all 0x55; vec[i] = i*0.1 - 3.0;
    # dotQ5_0 == dequant + scalar dot within 1e-3
    data = bytearray(44)
    data[0], data[1] = 0x00, 0x38
    data[2:6] = bytes([0xAA] * 4)
    for j in range(16):
        data[6 + j] = (j & 15) | (((j + 3) & 15) << 4)
    data[22], data[23] = 0x00, 0x30
    data[28:44] = bytes([0x55] * 16)
    vec = [np.float32(np.float32(i) * np.float32(0.1)) - np.float32(3.0) for i in range(64)]
    dec = [bits_to_f32(b) for b in q5_0_decode(bytes(data[:22])) + q5_0_decode(bytes(data[22:]))]
    exp = np.float32(0)
    for d, v in zip(dec, vec):
        exp = np.float32(exp + np.float32(np.float32(d) * v))
    return {"hex": data.hex(), "vec": [float(v) for v in vec], "expect": float(exp), "tol": 1e-3}


def dot_iq4_nl_case() -> dict:
    # dequant.zig:737-758: block 0 d=1, qs[i] = i | (15-i)<<4; block 1 d=2,
    # qs[i] = (i+3)&15 | ((i+5)&15)<<4; vec[i] = ((i % 7) + 1) * 0.25
    data = bytearray(36)
    data[0], data[1] = 0x00, 0x3C
    data[18], data[19] = 0x00, 0x40
    for i in range(16):
        data[2 + i] = (i & 15) | ((15 - i) << 4)
        data[20 + i] = ((i + 3) & 15) | (((i + 5) & 15) << 4)
    vec = [np.float32((i % 7) + 1) * np.float32(0.25) for i in range(64)]
    dec = [bits_to_f32(b) for b in iq4nl_decode(bytes(data[:18])) + iq4nl_decode(bytes(data[18:]))]
    exp = np.float32(0)
    for d, v in zip(dec, vec):
        exp = np.float32(exp + np.float32(np.float32(d) * v))
    return {"hex": data.hex(), "vec": [float(v) for v in vec], "expect": float(exp), "tol": 1e-3}


def q8_1_cases() -> list[dict]:
    cases = []
    # halves that round away from zero (d = 1 exactly: amax 127)
    x = np.zeros(32, np.float32)
    x[:8] = [127.0, 2.5, -3.5, 0.5, -0.5, 126.5, -126.5, 1.49]
    cases.append({"name": "q8_1_halves", "x": [float(v) for v in x], "hex": q8_1_quantize(x).hex()})
    cases.append({"name": "q8_1_zero_block", "x": [0.0] * 32, "hex": q8_1_quantize(np.zeros(32, np.float32)).hex()})
    rng = np.random.Generator(np.random.PCG64(20261203))
    x = rng.normal(0, 1.5, 96).astype(np.float32)
    cases.append({"name": "q8_1_random", "x": [float(v) for v in x], "hex": q8_1_quantize(x).hex()})
    return cases


def dot_q8_0_case() -> dict:
    # dequant.zig:680-700: block0 d=0.5 values 1..32, block1 d=0.25 values -16..15,
    # vec[i] = i*0.1 - 3.0 ; expected == dequant + scalar dot within 1e-3
    data = bytearray(68)
    data[0], data[1] = 0x00, 0x38
    for i in range(32):
        data[2 + i] = i + 1
    data[34], data[35] = 0x00, 0x34
    for i in range(32):
        data[36 + i] = (i - 16) & 0xFF
    vec = [np.float32(np.float32(i) * np.float32(0.1)) - np.float32(3.0) for i in range(64)]
    dec = [bits_to_f32(b) for b in q8_0_decode(bytes(data[:34])) + q8_0_decode(bytes(data[34:]))]
    exp = np.float32(0)
    for d, v in zip(dec, vec):
        exp = np.float32(exp + np.float32(np.float32(d) * v))
    return {"hex": data.hex(), "vec": [float(v) for v in vec], "expect": float(exp), "tol": 1e-3}


def router_cases() -> dict:
    c = {}
    # gemma4/forward.zig:823-829 — stable ties
    c["topk_ties"] = {"scores": [1.0, 4.0, 4.0, -2.0, 3.5, 4.0, 0.0], "k": 4, "expect": [1, 2, 5, 4]}
    # gemma4/forward.zig:831-845 — online denominator
    c["online_denominator"] = {"scores": [-3.0, 0.5, 7.0, 2.0, 6.5, -1.0], "k": 3}
    # gemma4/forward.zig:847-861
    c["softmax_topk"] = {"scores": [0.5, 4.0, -1.0, 2.5, 3.0, -0.25], "k": 3}
    # gemma4/forward.zig:863-891
    c["topk_matvec_6x5"] = {
        "weights": [1.0, -2.0, 0.5, 4.0, -1.0, 0.25, 3.0, 2.0, -0.5, 1.5, -1.0, 0.0, 0.0, 2.0, 3.0,
                    2.5, -1.5, 0.25, 0.0, 1.0, 0.0, 0.5, -2.0, 1.0, 2.0, 1.25, -0.25, 1.5, -2.0, 0.75],
        "rows": 6, "cols": 5, "vec": [0.5, -1.0, 2.0, 0.25, -0.75], "k": 3}
    # gemma4/forward.zig:893-922 — 37x33 deterministic weights, pool of 4
    c["par_37x33"] = {"rows": 37, "cols": 33, "k": 8,
                      "weights": [((i * 17 + 11) % 23 - 9) * 0.125 for i in range(37 * 33)],
                      "vec": [((i * 13 + 7) % 19 - 8) * 0.2 for i in range(33)], "threads": 4}
    # gemma4/forward.zig:924-960 — streamed 5x4 router, k=2
    c["streamed_5x4"] = {"rows": 5, "cols": 4, "k": 2,
                         "weights": [0.5, -1.0, 1.5, 0.25, 2.0, 0.0, -0.5, 1.0, -1.0, 2.0, 0.5, -0.25,
                                     1.25, -0.75, 0.0, 2.0, 0.0, 0.25, 1.0, -1.5],
                         "vec": [1.0, -0.5, 0.75, 2.0]}
    # src/gpu/matvec.zig:3582-3656 — d=8, E=4, k=2, router input 1 after the fused
    # RMS (x=1, scale sqrt(8)/sqrt(8)); rows 1 and 3 all ones, row 2 all 0.5,
    # expert scales {1,2,3,4} -> ids {1,3}, scales 2e^8/D, 4e^8/D, D = 2e^8+e^4+1
    D = 2 * np.exp(8.0) + np.exp(4.0) + 1.0
    w = [0.0] * 8 + [1.0] * 8 + [0.5] * 8 + [1.0] * 8
    c["gpu_router_closed_form"] = {"rows": 4, "cols": 8, "k": 2, "weights": w, "vec": [1.0] * 8,
                                   "expert_scale": [1.0, 2.0, 3.0, 4.0], "expect_ids": [1, 3],
                                   "expect_w": [2 * np.exp(8.0) / D, 4 * np.exp(8.0) / D], "tol": 1e-6}
    return c


def misc_cases() -> dict:
    return {
        # src/gpu/matvec.zig:3658-3727 and src/model/sample.zig:188-191
        "argmax": [{"values": [-4.0, 3.0, 9.0, 2.0, 9.0, 1.0], "expect": 2},
                   {"values": "1024x-4 with [17]=9,[900]=9", "n": 1024, "peaks": [17, 900], "expect": 17}],
        # src/ops/math.zig:173-191
        "quant_matvec_f32": {"rows": 3, "cols": 5,
                             "mat": [1.0, -2.0, 0.5, 4.0, -1.0, 0.25, 3.0, 2.0, -0.5, 1.5, -1.0, 0.0, 0.0, 2.0, 3.0],
                             "vec": [0.5, -1.0, 2.0, 0.25, -0.75], "tol": 1e-6},
        # src/ops/math.zig:344-354
        "rmsnorm": {"x": [1.0, 2.0, 3.0, 4.0], "w": [1.0] * 4, "eps": 1e-8,
                    "expect": [v / np.sqrt(7.5) for v in (1.0, 2.0, 3.0, 4.0)], "tol": 1e-5},
        # src/ops/math.zig:378-393
        "softmax": [{"x": [1.0, 2.0, 3.0], "tol": 1e-6}, {"x": [1000.0, 1001.0, 1002.0], "tol": 1e-5}],
        # src/ops/math.zig:401-413
        "dotf32_lengths": [1, 7, 8, 32, 33],
    }


def main() -> None:
    g = {"comment": "generated by tests/golden/gen_golden.py; f32 values stored as bit patterns",
         "dequant": dequant_cases(), "dot_q8_0": dot_q8_0_case(), "dot_q5_0": dot_q5_0_case(),
         "dot_iq4_nl": dot_iq4_nl_case(), "q8_1": q8_1_cases(), "router": router_cases(),
         "misc": misc_cases()}
    OUT.write_text(json.dumps(g, indent=1, default=float) + "\n")
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
