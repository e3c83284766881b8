"""The thin strips' count decomposition, exhaustively on the CPU: for every
pool row d, threshold v and window k,
    #{t < k : R[d][t] < v} = SW[d][v][k // 32].count
                             + popcount(SW[d][v][k // 32].word & (2^(k % 32) - 1))
with SW[d][v][w] = {stream word w of threshold v, #{t < 32 w : R[d][t] < v}}
(the table the stream-table kernel builds beside the stream words; word 0
at w = 2^p / 32)."""
import random

import numpy as np
import pytest

from scmp_vit_b200 import config_helpers as ch


def _strip_table(R: np.ndarray, T: int):
    D = R.shape[0]
    WT = max(T // 32, 1)
    words = np.zeros((D, T + 1, WT + 1), dtype=np.uint64)
    counts = np.zeros((D, T + 1, WT + 1), dtype=np.int64)
    for v in range(T + 1):
        bits = (R < v)  # [D, T]
        for w in range(WT):
            chunk = bits[:, 32 * w:32 * w + 32]
            words[:, v, w] = (chunk * (1 << np.arange(chunk.shape[1], dtype=np.uint64))).sum(1)
            counts[:, v, w + 1] = counts[:, v, w] + chunk.sum(1)
    return words, counts


@pytest.mark.parametrize("p", [4, 7, 8])
def test_prefix_count_decomposition(p):
    T = 1 << p
    random.seed(p)
    R = np.asarray(ch.make_sobol_simple_config(6, 6, p)["table"], dtype=np.int64)[:, :T]
    words, counts = _strip_table(R, T)
    for d in range(R.shape[0]):
        for v in range(T + 1):
            direct = np.concatenate([[0], np.cumsum(R[d] < v)])  # counts for k = 0 .. T
            for k in range(T + 1):
                w = k >> 5
                mask = (1 << (k & 31)) - 1
                word = int(words[d, v, w]) if w < max(T // 32, 1) else 0
                got = int(counts[d, v, w]) + bin(word & mask).count("1")
                assert got == direct[k], (d, v, k)
