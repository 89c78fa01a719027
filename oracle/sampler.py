"""CPU restatement of the reference's token samplers. Test infrastructure only.

Follows attnrank/src/model.cpp:
  GreedySampler::select    :70-73   the first index of the largest logit
  NucleusSampler::select   :79-122  top_k candidates by descending logit, weights
                                     exp((logit - max) / temperature) in double, the shortest
                                     prefix whose running share reaches top_p, a uniform draw in
                                     [0, prefix weight) walked down the prefix
  make_sampler             :124-127 temperature <= 0 -> greedy
The generator is std::mt19937_64 (seeded with config.seed, model.cpp:75), restated below from its
published definition (Matsumoto & Nishimura; the parameters the C++ standard fixes for
mt19937_64), and the draw is std::uniform_real_distribution<double>(0, w): one 64-bit output x
gives U = double(x) / 2^64 (std::generate_canonical with a 64-bit engine; a U that rounds to 1 is
replaced by the largest double below 1), and the draw is U * w.

Candidates are ordered here by (descending logit, ascending index). The reference orders them
with std::partial_sort, which leaves equal logits in an unspecified order; the two agree whenever
no tie decides the returned token, which is how the golden fixtures use this restatement.
"""
from __future__ import annotations

import math

import numpy as np

_MASK = (1 << 64) - 1


class MT19937_64:
    """The 64-bit Mersenne Twister (w=64, n=312, m=156, r=31)."""

    N, M = 312, 156
    MATRIX_A = 0xB5026F5AA96619E9
    UPPER, LOWER = 0xFFFFFFFF80000000, 0x7FFFFFFF

    def __init__(self, seed: int):
        self.state = [0] * self.N
        self.state[0] = seed & _MASK
        for i in range(1, self.N):
            previous = self.state[i - 1]
            self.state[i] = (6364136223846793005 * (previous ^ (previous >> 62)) + i) & _MASK
        self.index = self.N

    def _twist(self) -> None:
        s = self.state
        for i in range(self.N):
            y = (s[i] & self.UPPER) | (s[(i + 1) % self.N] & self.LOWER)
            value = s[(i + self.M) % self.N] ^ (y >> 1)
            if y & 1:
                value ^= self.MATRIX_A
            s[i] = value
        self.index = 0

    def next(self) -> int:
        if self.index >= self.N:
            self._twist()
        y = self.state[self.index]
        self.index += 1
        y ^= (y >> 29) & 0x5555555555555555
        y ^= (y << 17) & 0x71D67FFFEDA60000
        y ^= (y << 37) & 0xFFF7EEE000000000
        y ^= y >> 43
        return y & _MASK


def uniform(generator: MT19937_64, high: float) -> float:
    """std::uniform_real_distribution<double>(0, high) on a 64-bit engine."""
    unit = float(generator.next()) / 18446744073709551616.0  # float() rounds to nearest even
    if unit >= 1.0:
        unit = math.nextafter(1.0, 0.0)
    return unit * high


def greedy(logits: np.ndarray) -> int:
    return int(np.argmax(np.asarray(logits, dtype=np.float32)))  # first maximum


class Nucleus:
    def __init__(self, temperature: float, top_p: float, top_k: int, seed: int):
        if not temperature > 0.0:
            raise ValueError("nucleus sampling needs a positive temperature")
        # the config holds float temperature and top_p; the reference widens them to double
        self.temperature = float(np.float32(temperature))
        self.top_p = float(np.float32(top_p))
        self.top_k = int(top_k)
        self.generator = MT19937_64(int(seed))

    def select(self, logits: np.ndarray) -> int:
        values = np.asarray(logits, dtype=np.float32)
        if values.size == 0:
            raise ValueError("cannot sample from empty logits")
        order = np.lexsort((np.arange(values.size), -values.astype(np.float64)))
        keep = min(self.top_k, values.size) if self.top_k > 0 else values.size
        order = order[:keep]
        top = float(values[order[0]])
        weights = [math.exp((float(values[i]) - top) / self.temperature) for i in order]
        total = 0.0
        for w in weights:
            total += w
        nucleus = keep
        running = 0.0
        for i, w in enumerate(weights):
            running += w / total
            if running >= self.top_p:
                nucleus = i + 1
                break
        mass = 0.0
        for w in weights[:nucleus]:
            mass += w
        remaining = uniform(self.generator, mass)
        for i in range(nucleus):
            remaining -= weights[i]
            if remaining <= 0.0:
                return int(order[i])
        return int(order[nucleus - 1])


def make_sampler(temperature: float, top_p: float, top_k: int, seed: int):
    """make_sampler: an object with select(logits) -> token id."""
    if temperature <= 0.0:
        class _Greedy:
            @staticmethod
            def select(logits):
                return greedy(logits)
        return _Greedy()
    return Nucleus(temperature, top_p, top_k, seed)
