"""The nibble arithmetic of the e2m1 producers, checked exhaustively on the CPU.

The e2m1 kernels (tcgen05.mma kind::mxf4 with every block scale 1.0) take
operands in {-1, 0, +1} as e2m1 nibbles 0xA, 0x0, 0x2; nibble i (bits
4i .. 4i + 3) of a 32-bit word holds stream position 8 w + i of the word's
group.  These tests restate the producers' operations in numpy and check
them against the definitions over every input the kernels can see:

* window word: __funnelshift_lc(pattern, 0, max(4 (k - t0) - 32 w, 0)) must
  hold sigma in nibble i iff t0 + 8 w + i < k, for k - t0 in [-512, 1024]
  (every window length and every thread's first position) and both signs;
* stream word: two byte-SWAR compares u + PC against the even and odd
  positions' pool complements, sign-replicated, nibble-selected and masked,
  must hold sigma * [R >> shift < u] at every position, for every threshold
  u < 128 and pool byte R;
* pool complement layout: slot j of an 8-byte group holds position 2 j
  (j < 4) or 2 (j - 4) + 1, exactly what the stream word expects.
"""
import numpy as np

M32 = np.uint64(0xFFFFFFFF)
PAT = {1: 0x22222222, -1: 0xAAAAAAAA}  # e2m1 +1.0 / -1.0 in every nibble


def e2m1_value(nib):
    """{0x0, 0x2, 0xA} -> {0, +1, -1}; anything else is a failure."""
    table = {0x0: 0, 0x2: 1, 0xA: -1}
    return np.vectorize(lambda v: table.get(int(v), 99))(nib)


def nibbles_of(w):
    return [((w >> np.uint64(4 * i)) & np.uint64(0xF)) for i in range(8)]


def funnelshift_lc(lo, hi, shift):
    """__funnelshift_lc: (hi:lo) << min(shift, 32), the upper 32 bits."""
    s = np.minimum(shift, 32).astype(np.uint64)
    v = (np.uint64(hi) << np.uint64(32)) | np.uint64(lo)
    # python ints avoid the 64-bit overflow of the shifted concatenation
    return np.array([((int(v) << int(x)) >> 32) & 0xFFFFFFFF for x in s], dtype=np.uint64)


def test_window_words_exhaustive():
    rel = np.arange(-128, 257, dtype=np.int64)  # k - t0, positions
    k4 = 4 * rel
    for sign, pat in PAT.items():
        for w in range(16):
            shift = np.maximum(k4 - 32 * w, 0)
            word = funnelshift_lc(pat, 0, shift)
            for i, nib in enumerate(nibbles_of(word)):
                expect = sign * (8 * w + i < rel).astype(np.int64)
                np.testing.assert_array_equal(e2m1_value(nib), expect)


def sign_replicate(x):
    out = np.zeros_like(x)
    for byte in range(4):
        top = (x >> np.uint64(8 * byte + 7)) & np.uint64(1)
        out |= (top * np.uint64(0xFF)) << np.uint64(8 * byte)
    return out


def stream_word(u, pc_even, pc_odd, pat):
    e = sign_replicate((u * np.uint64(0x01010101) + pc_even) & M32)
    o = sign_replicate((u * np.uint64(0x01010101) + pc_odd) & M32)
    return ((e & np.uint64(0x0F0F0F0F)) | (o & np.uint64(0xF0F0F0F0))) & np.uint64(pat)


def test_stream_words_exhaustive():
    rng = np.random.default_rng(0)
    u = np.arange(0, 128, dtype=np.uint64)
    for shift in (0, 1):
        for sign, pat in PAT.items():
            for trial in range(24):
                R = rng.integers(0, 256 if shift else 128, size=8)  # positions 0..7 of a group
                Rs = R >> shift
                pc = (0x7F - Rs).astype(np.uint64)
                pc_even = pc[0] | (pc[2] << 8) | (pc[4] << 16) | (pc[6] << 24)
                pc_odd = pc[1] | (pc[3] << 8) | (pc[5] << 16) | (pc[7] << 24)
                word = stream_word(u, np.uint64(pc_even), np.uint64(pc_odd), pat)
                for i, nib in enumerate(nibbles_of(word)):
                    expect = sign * (Rs[i] < u.astype(np.int64)).astype(np.int64)
                    np.testing.assert_array_equal(e2m1_value(nib), expect)
    # every (threshold, pool byte) pair at one position, the others fixed
    for shift in (0, 1):
        for R0 in range(256 if shift else 128):
            R = np.array([R0, 5, 77, 126, 0, 127, 64, 33]) if not shift else \
                np.array([R0, 10, 154, 252, 0, 255, 128, 66])
            Rs = R >> shift
            pc = (0x7F - Rs).astype(np.uint64)
            pc_even = pc[0] | (pc[2] << 8) | (pc[4] << 16) | (pc[6] << 24)
            pc_odd = pc[1] | (pc[3] << 8) | (pc[5] << 16) | (pc[7] << 24)
            word = stream_word(u, np.uint64(pc_even), np.uint64(pc_odd), PAT[1])
            nib0 = nibbles_of(word)[0]
            np.testing.assert_array_equal(e2m1_value(nib0),
                                          (Rs[0] < u.astype(np.int64)).astype(np.int64))


def test_pool_complement_nibble_pair_layout():
    """The slot -> position map of pool_complement_kernel (nibble_pairs) puts
    positions (0, 2, 4, 6) in the first word and (1, 3, 5, 7) in the second
    of every 8-byte group, for every padded stream length."""
    for lp in (128, 256):
        slot = np.arange(lp)
        pos = (slot & ~7) + (((slot & 3) << 1) | ((slot >> 2) & 1))
        assert sorted(pos.tolist()) == list(range(lp))  # a permutation
        for g in range(lp // 8):
            even = pos[8 * g: 8 * g + 4]
            odd = pos[8 * g + 4: 8 * g + 8]
            np.testing.assert_array_equal(even, 8 * g + np.array([0, 2, 4, 6]))
            np.testing.assert_array_equal(odd, 8 * g + np.array([1, 3, 5, 7]))
