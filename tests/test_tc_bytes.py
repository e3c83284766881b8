"""The byte arithmetic the tensor-core row producers use, checked
exhaustively on the CPU.

A producer writes four stream bytes with one 32-bit multiply-add, one
sign-replicating byte permute (prmt 0xBA98) and one AND.  These tests restate
those three operations in numpy and check them against the definitions over
every input the kernel can see:

* enable window: byte b of word j of a chunk starting at stream position
  t0 = t0A + 16 i must be sigma * [t0 + 4 j + b < k], for every window length
  k <= 128 (Lp <= 128, or one half of Lp = 256), every chunk and sign;
* stream: byte b must be sigma * [R >> shift < u] for every threshold u < 128
  and pool byte R (shift 1 for bipolar p = 8), with the pool complement
  0x7F - (R >> shift) as the addend.
"""
import numpy as np

REP = np.uint64(0x01010101)
M32 = np.uint64(0xFFFFFFFF)
TW = [0x03020100, 0x07060504, 0x0B0A0908, 0x0F0E0D0C]


def mad(a, b, c):
    """mad.lo.u32 on uint64 carriers."""
    return (a.astype(np.uint64) * np.uint64(b) + c.astype(np.uint64)) & M32


def sign_replicate(x):
    """prmt.b32 x, 0, 0xBA98: each byte becomes 0xFF if its top bit is set."""
    out = np.zeros_like(x)
    for byte in range(4):
        top = (x >> np.uint64(8 * byte + 7)) & np.uint64(1)
        out |= (top * np.uint64(0xFF)) << np.uint64(8 * byte)
    return out


def bytes_of(w):
    return [((w >> np.uint64(8 * b)) & np.uint64(0xFF)).astype(np.int64) for b in range(4)]


def to_s8(v):
    return np.where(v >= 128, v - 256, v)


def test_enable_window_bytes_exhaustive():
    k = np.arange(0, 129, dtype=np.int64)
    for sign in (1, -1):
        sm = np.uint64(0x01010101 if sign > 0 else 0xFFFFFFFF)
        for t0a in (0, 64):                      # 64 * hA (Lp >= 128); 0 for Lp = 64
            kbase = ((k - t0a) & 0xFFFFFFFF).astype(np.uint64)
            for i in range(4):
                for j in range(4):
                    base = (0x7F7F7F7F - 0x10101010 * i - TW[j]) & 0xFFFFFFFF
                    w = sign_replicate(mad(kbase, REP, np.full_like(kbase, base))) & sm
                    for b, v in enumerate(bytes_of(w)):
                        t = t0a + 16 * i + 4 * j + b
                        np.testing.assert_array_equal(to_s8(v), sign * (t < k).astype(np.int64))


def test_stream_bytes_exhaustive():
    u_all = np.arange(0, 128, dtype=np.int64)
    R = np.arange(0, 256, dtype=np.int64)
    for shift in (0, 1):
        Rs = R if shift else R[:128]             # p <= 7 pools hold bytes < 128
        comp = 0x7F - (Rs >> shift)              # pool complement byte
        for sign in (1, -1):
            sm = np.uint64(0x01010101 if sign > 0 else 0xFFFFFFFF)
            for u in u_all:
                # the pool byte under test in position b, a neighbour beside it
                for b in range(4):
                    word = (comp.astype(np.uint64) << np.uint64(8 * b)) | \
                        (np.uint64(0x7F) << np.uint64(8 * ((b + 1) % 4)))
                    w = sign_replicate(mad(np.full(len(Rs), u, np.int64).astype(np.uint64),
                                           REP, word)) & sm
                    got = to_s8(bytes_of(w)[b])
                    np.testing.assert_array_equal(got, sign * ((Rs >> shift) < u).astype(np.int64))


def test_bipolar_p8_shift_is_exact():
    """Bipolar codes are even (c = 2|x|), so [R < |c|] == [R >> 1 < |c| >> 1]."""
    R = np.arange(256)[:, None]
    c = np.arange(0, 256, 2)[None, :]
    np.testing.assert_array_equal(R < c, (R >> 1) < (c >> 1))
