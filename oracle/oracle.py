"""ctypes/numpy wrapper of the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
bench.py may import this module; the product library never does.  See
oracle/ckks_oracle.h for what the oracle restates, which reference lines it
follows, and its parity status (bit-level parity with Phantom is unpinned;
primes, partition math and decode-level semantics are pinned).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "libckks_oracle.so")
_lib = None

u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")
i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (g++, OpenMP)."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_LIB_PATH)
        V, P, I, U32, U64, D = None, C.c_void_p, C.c_int, C.c_uint32, C.c_uint64, C.c_double
        sig = {
            "ork_gen_primes": (I, [U32, i32p, I, u64p]),
            "ork_is_prime": (I, [U64]),
            "ork_create": (P, [U32, u64p, I, u64p, I]),
            "ork_destroy": (V, [P]),
            "ork_set_threads": (V, [I]),
            "ork_get_threads": (I, []),
            "ork_num_digits": (I, [P, I]),
            "ork_psi": (U64, [P, I]),
            "ork_ntt_forward": (V, [P, u64p, I, i32p]),
            "ork_ntt_inverse": (V, [P, u64p, I, i32p]),
            "ork_galois_elt": (U32, [P, I]),
            "ork_galois_ntt": (V, [P, U32, u64p, u64p, I]),
            "ork_galois_coeff": (V, [P, U32, u64p, u64p, I, i32p]),
            "ork_bconv": (V, [P, u64p, i32p, I, u64p, i32p, I]),
            "ork_modup": (V, [P, u64p, I, u64p]),
            "ork_inner_product": (V, [P, u64p, I, u64p, u64p]),
            "ork_moddown": (V, [P, u64p, I, u64p]),
            "ork_keyswitch": (V, [P, u64p, I, u64p, u64p]),
            "ork_apply_galois": (V, [P, u64p, I, U32, u64p, u64p]),
            "ork_relinearize": (V, [P, u64p, I, u64p, u64p]),
            "ork_rotate_hoisted": (V, [P, u64p, I, I, C.POINTER(C.c_uint32), C.POINTER(C.c_void_p), u64p]),
            "ork_linear_transform_hoisted": (V, [P, u64p, I, I, C.POINTER(C.c_uint32),
                                                 C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                                 u64p]),
            "ork_bsgs_matmul": (V, [P, C.POINTER(C.c_void_p), I, I, I, I, I, I,
                                    C.POINTER(C.c_uint32), C.POINTER(C.c_void_p),
                                    C.POINTER(C.c_uint32), C.POINTER(C.c_void_p),
                                    C.POINTER(C.c_void_p), I, C.POINTER(C.c_void_p)]),
            "ork_encode_basis": (V, [P, f64p, f64p, I, D, i32p, I, u64p]),
            "ork_rescale": (V, [P, u64p, I, u64p]),
            "ork_prng": (U64, [U64, U64, U64]),
            "ork_gauss": (I, [U64]),
            "ork_gauss_table": (V, [u64p]),
            "ork_secret": (V, [P, U64, I, i8p]),
            "ork_secret_ntt": (V, [P, i8p, I, u64p]),
            "ork_keygen_galois": (V, [P, i8p, U32, U64, u64p]),
            "ork_keygen_relin": (V, [P, i8p, U64, u64p]),
            "ork_encode": (V, [P, f64p, f64p, I, D, I, u64p]),
            "ork_decode": (V, [P, u64p, I, D, f64p, f64p, I]),
            "ork_encrypt": (V, [P, i8p, u64p, I, U64, u64p]),
            "ork_decrypt": (V, [P, i8p, u64p, I, I, u64p]),
            "ork_multiply": (V, [P, u64p, u64p, I, u64p]),
            "ork_ks_noise_log2": (D, [P, i8p, u64p, u64p, u64p, I]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def gen_primes(log_n: int, bit_sizes) -> np.ndarray:
    bits = np.ascontiguousarray(bit_sizes, dtype=np.int32)
    out = np.zeros(len(bits), dtype=np.uint64)
    if lib().ork_gen_primes(log_n, bits, len(bits), out) != 0:
        raise ValueError("not enough primes")
    return out


def set_threads(n: int) -> None:
    lib().ork_set_threads(int(n))


def prng(seed: int, domain: int, idx: int) -> int:
    return int(lib().ork_prng(seed, domain, idx))


class Oracle:
    """One parameter set: N = 2^log_n, L Q primes, alpha P primes."""

    def __init__(self, log_n: int, q, p):
        self.log_n = int(log_n)
        self.N = 1 << self.log_n
        self.q = np.ascontiguousarray(q, dtype=np.uint64)
        self.p = np.ascontiguousarray(p, dtype=np.uint64)
        self.L, self.alpha = len(self.q), len(self.p)
        self.h = lib().ork_create(self.log_n, self.q, self.L, self.p, self.alpha)
        self.moduli = np.concatenate([self.q, self.p])

    def __del__(self):
        h = getattr(self, "h", None)
        if h and _lib is not None:
            _lib.ork_destroy(h)
            self.h = None

    # -- helpers -------------------------------------------------------------
    def digits(self, Ql: int) -> int:
        return int(lib().ork_num_digits(self.h, Ql))

    def key_words(self) -> int:
        return self.digits(self.L) * 2 * (self.L + self.alpha) * self.N

    def psi(self, k: int) -> int:
        return int(lib().ork_psi(self.h, k))

    def galois_elt(self, step: int) -> int:
        return int(lib().ork_galois_elt(self.h, int(step)))

    # -- transforms ----------------------------------------------------------
    def ntt(self, data: np.ndarray, key_idx, inverse: bool = False) -> np.ndarray:
        a = np.ascontiguousarray(data, dtype=np.uint64).copy()
        idx = np.ascontiguousarray(key_idx, dtype=np.int32)
        n = a.size // self.N
        assert len(idx) == n
        f = lib().ork_ntt_inverse if inverse else lib().ork_ntt_forward
        f(self.h, a.reshape(-1), n, idx)
        return a

    def galois_ntt(self, data: np.ndarray, elt: int) -> np.ndarray:
        a = np.ascontiguousarray(data, dtype=np.uint64)
        out = np.empty_like(a)
        lib().ork_galois_ntt(self.h, elt, a.reshape(-1), out.reshape(-1), a.size // self.N)
        return out

    def galois_coeff(self, data: np.ndarray, elt: int, key_idx) -> np.ndarray:
        a = np.ascontiguousarray(data, dtype=np.uint64)
        out = np.empty_like(a)
        idx = np.ascontiguousarray(key_idx, dtype=np.int32)
        lib().ork_galois_coeff(self.h, elt, a.reshape(-1), out.reshape(-1), a.size // self.N, idx)
        return out

    def bconv(self, x: np.ndarray, in_idx, out_idx) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.uint64)
        ii = np.ascontiguousarray(in_idx, dtype=np.int32)
        oi = np.ascontiguousarray(out_idx, dtype=np.int32)
        out = np.zeros((len(oi), self.N), dtype=np.uint64)
        lib().ork_bconv(self.h, x.reshape(-1), ii, len(ii), out.reshape(-1), oi, len(oi))
        return out

    # -- key switching -------------------------------------------------------
    def modup(self, c: np.ndarray, Ql: int) -> np.ndarray:
        c = np.ascontiguousarray(c, dtype=np.uint64)
        t = np.zeros((self.digits(Ql), Ql + self.alpha, self.N), dtype=np.uint64)
        lib().ork_modup(self.h, c.reshape(-1), Ql, t.reshape(-1))
        return t

    def inner_product(self, t: np.ndarray, Ql: int, key: np.ndarray) -> np.ndarray:
        cx = np.zeros((2, Ql + self.alpha, self.N), dtype=np.uint64)
        lib().ork_inner_product(self.h, np.ascontiguousarray(t).reshape(-1), Ql,
                                np.ascontiguousarray(key).reshape(-1), cx.reshape(-1))
        return cx

    def moddown(self, cx_poly: np.ndarray, Ql: int) -> np.ndarray:
        out = np.zeros((Ql, self.N), dtype=np.uint64)
        lib().ork_moddown(self.h, np.ascontiguousarray(cx_poly).reshape(-1), Ql, out.reshape(-1))
        return out

    def keyswitch(self, c: np.ndarray, Ql: int, key: np.ndarray) -> np.ndarray:
        out = np.zeros((2, Ql, self.N), dtype=np.uint64)
        lib().ork_keyswitch(self.h, np.ascontiguousarray(c).reshape(-1), Ql,
                            np.ascontiguousarray(key).reshape(-1), out.reshape(-1))
        return out

    def apply_galois(self, ct: np.ndarray, Ql: int, elt: int, key: np.ndarray) -> np.ndarray:
        out = np.zeros((2, Ql, self.N), dtype=np.uint64)
        lib().ork_apply_galois(self.h, np.ascontiguousarray(ct).reshape(-1), Ql, elt,
                               np.ascontiguousarray(key).reshape(-1), out.reshape(-1))
        return out

    def rotate(self, ct: np.ndarray, Ql: int, step: int, key: np.ndarray) -> np.ndarray:
        return self.apply_galois(ct, Ql, self.galois_elt(step), key)

    def relinearize(self, ct3: np.ndarray, Ql: int, key: np.ndarray) -> np.ndarray:
        out = np.zeros((2, Ql, self.N), dtype=np.uint64)
        lib().ork_relinearize(self.h, np.ascontiguousarray(ct3).reshape(-1), Ql,
                              np.ascontiguousarray(key).reshape(-1), out.reshape(-1))
        return out

    def rotate_hoisted(self, ct: np.ndarray, Ql: int, elts, keys) -> np.ndarray:
        n = len(elts)
        out = np.zeros((n, 2, Ql, self.N), dtype=np.uint64)
        e = (C.c_uint32 * n)(*[int(x) for x in elts])
        ks = [np.ascontiguousarray(k) for k in keys]
        kp = (C.c_void_p * n)(*[k.ctypes.data for k in ks])
        lib().ork_rotate_hoisted(self.h, np.ascontiguousarray(ct).reshape(-1), Ql, n, e, kp,
                                 out.reshape(-1))
        return out

    def linear_transform_hoisted(self, ct: np.ndarray, Ql: int, elts, keys, diags) -> np.ndarray:
        """sum_r diags[r] * rot_r(ct) with one ModUp and one ModDown; diags[r]:
        [Ql + alpha][N] NTT-form plaintexts in the extended basis."""
        n = len(elts)
        out = np.zeros((2, Ql, self.N), dtype=np.uint64)
        e = (C.c_uint32 * n)(*[int(x) for x in elts])
        ks = [np.ascontiguousarray(k) for k in keys]
        ds = [np.ascontiguousarray(d, dtype=np.uint64) for d in diags]
        for d in ds:
            assert d.shape == (Ql + self.alpha, self.N)
        kp = (C.c_void_p * n)(*[k.ctypes.data for k in ks])
        dp = (C.c_void_p * n)(*[d.ctypes.data for d in ds])
        lib().ork_linear_transform_hoisted(self.h, np.ascontiguousarray(ct).reshape(-1), Ql, n,
                                           e, kp, dp, out.reshape(-1))
        return out

    def bsgs_matmul(self, xs, Ql: int, unit: int, B: int, G: int, pts, keys,
                    g_range=None, n_out: int | None = None) -> np.ndarray:
        """Block BSGS matrix product (ork_bsgs_matmul): xs [n_in] ciphertexts
        [2][Ql][N]; pts[((o n_in + i) G + g) B + b] [Ql][N] NTT-form diagonals;
        keys: {step: galois key} for steps b*unit (0 < b < B) and g*B*unit
        (g > 0).  Returns y [n_out][2][Ql][N]."""
        n_in = len(xs)
        g_lo, g_hi = g_range if g_range is not None else (0, G)
        if n_out is None:
            n_out = len(pts) // (n_in * G * B)
        assert len(pts) == n_out * n_in * G * B
        xa = [np.ascontiguousarray(x, dtype=np.uint64) for x in xs]
        pa = [np.ascontiguousarray(p, dtype=np.uint64) for p in pts]
        for x in xa:
            assert x.shape == (2, Ql, self.N)
        for p in pa:
            assert p.shape == (Ql, self.N)
        be = (C.c_uint32 * max(B - 1, 1))(*[self.galois_elt(b * unit) for b in range(1, B)])
        bk = [np.ascontiguousarray(keys[b * unit]) for b in range(1, B)]
        bkp = (C.c_void_p * max(B - 1, 1))(*[k.ctypes.data for k in bk])
        ge = (C.c_uint32 * G)(*[self.galois_elt(g * B * unit) if g else 0 for g in range(G)])
        gk = [np.ascontiguousarray(keys[g * B * unit]) if g_lo <= g < g_hi and g else None
              for g in range(G)]
        gkp = (C.c_void_p * G)(*[k.ctypes.data if k is not None else None for k in gk])
        y = np.zeros((n_out, 2, Ql, self.N), dtype=np.uint64)
        xp = (C.c_void_p * n_in)(*[x.ctypes.data for x in xa])
        pp = (C.c_void_p * len(pa))(*[p.ctypes.data for p in pa])
        yp = (C.c_void_p * n_out)(*[y[o].ctypes.data for o in range(n_out)])
        lib().ork_bsgs_matmul(self.h, xp, n_in, Ql, B, G, g_lo, g_hi, be, bkp, ge, gkp, pp,
                              n_out, yp)
        return y

    def rescale(self, ct: np.ndarray, Ql: int) -> np.ndarray:
        """[2][Ql][N] -> [2][Ql-1][N]: divide by q_{Ql-1} and round."""
        out = np.zeros((2, Ql - 1, self.N), dtype=np.uint64)
        lib().ork_rescale(self.h, np.ascontiguousarray(ct).reshape(-1), Ql, out.reshape(-1))
        return out

    # -- keys, encoding, encryption -------------------------------------------
    def secret(self, seed: int, hamming_weight: int = 0) -> np.ndarray:
        s = np.zeros(self.N, dtype=np.int8)
        lib().ork_secret(self.h, seed, hamming_weight, s)
        return s

    def secret_ntt(self, s: np.ndarray, n_limbs: int) -> np.ndarray:
        out = np.zeros((n_limbs, self.N), dtype=np.uint64)
        lib().ork_secret_ntt(self.h, s, n_limbs, out.reshape(-1))
        return out

    def keygen_galois(self, s: np.ndarray, elt: int, seed: int) -> np.ndarray:
        key = np.zeros((self.digits(self.L), 2, self.L + self.alpha, self.N), dtype=np.uint64)
        lib().ork_keygen_galois(self.h, s, elt, seed, key.reshape(-1))
        return key

    def keygen_relin(self, s: np.ndarray, seed: int) -> np.ndarray:
        key = np.zeros((self.digits(self.L), 2, self.L + self.alpha, self.N), dtype=np.uint64)
        lib().ork_keygen_relin(self.h, s, seed, key.reshape(-1))
        return key

    def encode(self, z: np.ndarray, scale: float, Ql: int) -> np.ndarray:
        z = np.asarray(z)
        re = np.ascontiguousarray(z.real, dtype=np.float64)
        im = np.ascontiguousarray(np.imag(z) if np.iscomplexobj(z) else np.zeros(len(z)),
                                  dtype=np.float64)
        pt = np.zeros((Ql, self.N), dtype=np.uint64)
        lib().ork_encode(self.h, re, im, len(re), scale, Ql, pt.reshape(-1))
        return pt

    def encode_basis(self, z: np.ndarray, scale: float, key_idx) -> np.ndarray:
        """encode() into the key-basis primes key_idx (Q primes first, then P)."""
        z = np.asarray(z)
        re = np.ascontiguousarray(z.real, dtype=np.float64)
        im = np.ascontiguousarray(np.imag(z) if np.iscomplexobj(z) else np.zeros(len(z)),
                                  dtype=np.float64)
        idx = np.ascontiguousarray(key_idx, dtype=np.int32)
        pt = np.zeros((len(idx), self.N), dtype=np.uint64)
        lib().ork_encode_basis(self.h, re, im, len(re), scale, idx, len(idx), pt.reshape(-1))
        return pt

    def decode(self, pt: np.ndarray, Ql: int, scale: float, n_slots: int | None = None) -> np.ndarray:
        n = n_slots or self.N // 2
        re = np.zeros(n)
        im = np.zeros(n)
        lib().ork_decode(self.h, np.ascontiguousarray(pt).reshape(-1), Ql, scale, re, im, n)
        return re + 1j * im

    def encrypt(self, s: np.ndarray, pt: np.ndarray, Ql: int, seed: int) -> np.ndarray:
        ct = np.zeros((2, Ql, self.N), dtype=np.uint64)
        lib().ork_encrypt(self.h, s, np.ascontiguousarray(pt).reshape(-1), Ql, seed, ct.reshape(-1))
        return ct

    def decrypt(self, s: np.ndarray, ct: np.ndarray, Ql: int) -> np.ndarray:
        ct = np.ascontiguousarray(ct)
        pt = np.zeros((Ql, self.N), dtype=np.uint64)
        lib().ork_decrypt(self.h, s, ct.reshape(-1), ct.shape[0], Ql, pt.reshape(-1))
        return pt

    def multiply(self, a: np.ndarray, b: np.ndarray, Ql: int) -> np.ndarray:
        out = np.zeros((3, Ql, self.N), dtype=np.uint64)
        lib().ork_multiply(self.h, np.ascontiguousarray(a).reshape(-1),
                           np.ascontiguousarray(b).reshape(-1), Ql, out.reshape(-1))
        return out

    def ks_noise_log2(self, s, c_in, snew_ntt, ks, Ql) -> float:
        return float(lib().ork_ks_noise_log2(self.h, s, np.ascontiguousarray(c_in).reshape(-1),
                                              np.ascontiguousarray(snew_ntt).reshape(-1),
                                              np.ascontiguousarray(ks).reshape(-1), Ql))
