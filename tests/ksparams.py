"""Parameter sets shared by the tests (BASELINE configs 1-3 and small cases)."""
import functools

import numpy as np

from oracle.oracle import Oracle, gen_primes


@functools.lru_cache(maxsize=None)
def primes(log_n, bits):
    return gen_primes(log_n, list(bits))


# config 1: N=2^13, Q={60,40,40}, P={60}  (reference ckks_bench.txt:35 modulus)
CFG1 = dict(log_n=13, qbits=(60, 40, 40), pbits=(60,))
# config 3: N=2^16, Q = 58 + 34x42, P = 5x60, alpha = 5, dnum = 7
CFG3 = dict(log_n=16, qbits=(58,) + (42,) * 34, pbits=(60,) * 5)
# small multi-digit case: N=2^12, 7 Q primes, alpha=3 (3 digits, the last short)
SMALL = dict(log_n=12, qbits=(50,) + (40,) * 6, pbits=(55,) * 3)
# the reference's own correctness test: N=8192, bit sizes {60,40,40,40,60}, the
# last prime special (src/benchmarks/multi_gpu_keyswitch_test.cu:186-195)
REFTEST = dict(log_n=13, qbits=(60, 40, 40, 40), pbits=(60,))
# the other ring sizes of the reference's published correctness table
# (N = 16384; and 32768): column pass of 2^7 points
N14 = dict(log_n=14, qbits=(50, 40, 40, 40), pbits=(55, 55))
N15 = dict(log_n=15, qbits=(55,) + (40,) * 4, pbits=(58, 58, 58))
# one special prime, so every Q prime is a digit: 34 digits, more than the 32
# products the inner product sums before it reduces its accumulators
MANYDIG = dict(log_n=12, qbits=(50,) + (40,) * 33, pbits=(55,))


def split(cfg):
    pr = primes(cfg["log_n"], tuple(cfg["qbits"]) + tuple(cfg["pbits"]))
    L = len(cfg["qbits"])
    return cfg["log_n"], pr[:L], pr[L:]


@functools.lru_cache(maxsize=None)
def oracle_for(name):
    cfg = {"cfg1": CFG1, "cfg3": CFG3, "small": SMALL, "reftest": REFTEST, "n14": N14,
           "n15": N15, "manydig": MANYDIG}[name]
    log_n, q, p = split(cfg)
    return Oracle(log_n, q, p)


def random_limbs(moduli, n_limbs_each, N, seed):
    rng = np.random.default_rng(seed)
    out = np.empty((len(moduli), N), dtype=np.uint64)
    for i, q in enumerate(moduli):
        out[i] = rng.integers(0, int(q), size=N, dtype=np.uint64)
    return out


def reference_test_values(n, seed):
    """The reference test's input distribution, (rand() % 1000) / 100 - 5
    (multi_gpu_keyswitch_test.cu:211-215), drawn from a seeded generator."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 1000, size=n) / 100.0 - 5.0
