"""The reference's token sampler and the counter-based generator of the device sampler
(oracle, test infrastructure only).

* ``sample_distribution`` restates ``sample_topk`` (``src/moss_tts/_runtime/llm.py:10-19``)
  as the distribution it draws from: ``x = float32(logit) / T``, the ``top_k`` largest
  (descending; equal values in ascending index order), ``softmax`` over them in fp32, entries
  with ``cumsum - p > top_p`` removed, the rest in proportion to their probabilities
  (``torch.multinomial``). ``T <= 0`` is the argmax.
* ``philox4x32_10`` is the counter-based generator of Salmon, Moraes, Dror and Shaw,
  "Parallel random numbers: as easy as 1, 2, 3" (SC'11), checked against the published
  known-answer vectors of that paper's Random123 distribution.
* ``device_pick`` replays the device sampler's draw (``mt_heads_sample``): the uniform
  ``(philox(channel, position)[0] >> 8) * 2^-24`` times the kept mass, walked along the kept
  probabilities in order.
"""
import numpy as np

M0, M1 = 0xD2511F53, 0xCD9E8D57
W0, W1 = 0x9E3779B9, 0xBB67AE85
MASK = 0xFFFFFFFF


def philox4x32_10(counter, key):
    """Philox4x32 with 10 rounds; ``counter`` four and ``key`` two 32-bit ints."""
    c0, c1, c2, c3 = (int(v) & MASK for v in counter)
    k0, k1 = (int(v) & MASK for v in key)
    for _ in range(10):
        p0, p1 = M0 * c0, M1 * c2
        c0, c1, c2, c3 = ((p1 >> 32) ^ c1 ^ k0) & MASK, p1 & MASK, ((p0 >> 32) ^ c3 ^ k1) & MASK, p0 & MASK
        k0, k1 = (k0 + W0) & MASK, (k1 + W1) & MASK
    return c0, c1, c2, c3


def sample_distribution(logits, temperature, top_k, top_p):
    """``(indices, probabilities)`` of the tokens ``sample_topk`` can return and their
    probabilities (summing to 1), for one row of logits (float32 values)."""
    x = np.asarray(logits, dtype=np.float32)
    if not temperature > 0:
        return np.array([int(np.argmax(x))]), np.array([1.0])
    v = (x / np.float32(temperature)).astype(np.float32)
    k = min(int(top_k), v.shape[0])
    order = np.lexsort((np.arange(v.shape[0]), -v.astype(np.float64)))[:k]
    vals = v[order]
    e = np.exp((vals - vals[0]).astype(np.float32)).astype(np.float32)
    p = (e / e.sum(dtype=np.float32)).astype(np.float32)
    excl = (np.cumsum(p, dtype=np.float32) - p).astype(np.float32)
    keep = ~(excl > np.float32(top_p))
    q = np.where(keep, p, np.float32(0)).astype(np.float64)
    return order[keep], q[keep] / q.sum()


def device_pick(logits, temperature, top_k, top_p, seed, position, channel):
    """The index the device sampler draws for this (seed, position, channel), and the distance
    of its uniform target from the nearest boundary of the kept cumulative probabilities
    (fp32 rounding of the softmax can move a target that close to a boundary)."""
    idx, q = sample_distribution(logits, temperature, top_k, top_p)
    if len(idx) == 1:
        return int(idx[0]), 1.0
    r = philox4x32_10((channel + 1, position & MASK, (position >> 32) & MASK, 0), (seed & MASK, (seed >> 32) & MASK))
    u = (r[0] >> 8) * 2.0 ** -24
    edges = np.cumsum(q)
    pos = int(np.searchsorted(edges, u, side="right"))
    pos = min(pos, len(idx) - 1)
    return int(idx[pos]), float(np.min(np.abs(edges[:-1] - u))) if len(edges) > 1 else 1.0
