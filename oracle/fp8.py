"""FP8 e4m3 (``float8_e4m3fn``) helpers in plain numpy. Test infrastructure only.

e4m3fn: 1 sign bit, 4 exponent bits (bias 7), 3 mantissa bits, no infinities,
0x7F / 0xFF are NaN, largest finite magnitude 448. These helpers restate the
format from its definition (OCP 8-bit floating point spec), independent of
torch's own conversion, so the oracle does not lean on the library it checks.
"""
import numpy as np


def _decode_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        sign = -1.0 if b & 0x80 else 1.0
        exp = (b >> 3) & 0xF
        man = b & 0x7
        if exp == 0xF and man == 0x7:
            t[b] = np.nan
        elif exp == 0:
            t[b] = sign * (man / 8.0) * 2.0 ** -6
        else:
            t[b] = sign * (1.0 + man / 8.0) * 2.0 ** (exp - 7)
    return t


E4M3_TABLE = _decode_table()


def e4m3_to_f32(raw: np.ndarray) -> np.ndarray:
    """Decode e4m3 bytes (uint8 array of any shape) to float32."""
    return E4M3_TABLE[np.asarray(raw, dtype=np.uint8)]


def round_e4m3(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest e4m3 value (ties to even), saturating at 448.

    Matches ``cvt.rn.satfinite.e4m3x2.f32``: magnitudes beyond 448 clamp to 448.
    Returns float32 values that are exactly representable in e4m3.
    """
    x = np.asarray(x, dtype=np.float32)
    ax = np.abs(x).astype(np.float64)
    _, e = np.frexp(ax)
    expo = np.maximum(e - 1, -6)          # normal binade exponent, subnormals share 2^-6
    quantum = np.ldexp(1.0, expo - 3)     # 3 mantissa bits
    q = np.round(ax / quantum) * quantum  # numpy rounds half to even
    q = np.minimum(q, 448.0)
    return (np.sign(x) * q).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (ties to even); returns the uint16 bit patterns."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
