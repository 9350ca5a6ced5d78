"""Regenerates the golden fixtures in this directory from the reference tree.

Run here (where the read-only reference is mounted); the GPU box never reads
the reference, it uses the committed JSON files.

  python tests/golden/make_golden.py [/path/to/reference]

prime_kat.json      every (N, bit sizes) -> primes block that the reference's
                    Phantom CoeffModulus::Create printed in its L4 baseline run
                    (experiments/results/2026-03-29_l4_baseline-ops/raw/ckks_bench.txt)
partition_ref.json  outputs of the reference's own partition functions
                    (src/multi_gpu/partition/rns_partition.cuh:29-107), computed by
                    the library oracle/_ref/libref_partition.so built from those sources
"""
import ctypes as C
import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def prime_kat(ref):
    path = os.path.join(ref, "experiments/results/2026-03-29_l4_baseline-ops/raw/ckks_bench.txt")
    text = open(path).read().splitlines()
    out = []
    i = 0
    while i < len(text):
        m = re.search(r"poly_modulus_degree:\s*(\d+)", text[i])
        if m:
            n = int(m.group(1))
            bits_line = text[i + 1]
            bm = re.search(r"\(([\d +]+)\) bits", bits_line)
            bits = [int(b) for b in bm.group(1).split("+")]
            # the primes line follows after a blank line
            j = i + 2
            while j < len(text) and not re.match(r"^\s*\d{6,}", text[j]):
                j += 1
            primes = [int(x) for x in re.findall(r"\d+", text[j])]
            assert len(primes) == len(bits), (n, bits, primes)
            out.append({"N": n, "log_n": n.bit_length() - 1, "bits": bits, "primes": primes,
                        "source": "ckks_bench.txt:%d-%d" % (i + 1, j + 1)})
            i = j
        i += 1
    return out


def partition_ref():
    lib = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_partition.so"))
    sz = C.c_size_t
    lib.ref_owner_of_limb.restype = C.c_int
    lib.ref_owner_of_limb.argtypes = [sz, C.c_int]
    lib.ref_local_index_of_limb.restype = sz
    lib.ref_local_index_of_limb.argtypes = [sz, C.c_int]
    lib.ref_global_limb_index.restype = sz
    lib.ref_global_limb_index.argtypes = [C.c_int, sz, C.c_int]
    lib.ref_n_local_limbs.restype = sz
    lib.ref_n_local_limbs.argtypes = [C.c_int, C.c_int, sz]
    lib.ref_local_buf_offset.restype = sz
    lib.ref_local_buf_offset.argtypes = [sz, sz, sz, sz]
    lib.ref_global_buf_offset.restype = sz
    lib.ref_global_buf_offset.argtypes = [sz, sz, sz, sz]
    cases = []
    for G in (1, 2, 3, 4, 8):
        for total in (0, 1, 3, 5, 20, 35, 36, 40):
            rec = {"G": G, "total": total,
                   "owner": [lib.ref_owner_of_limb(j, G) for j in range(total)],
                   "local_index": [lib.ref_local_index_of_limb(j, G) for j in range(total)],
                   "n_local": [lib.ref_n_local_limbs(g, G, total) for g in range(G)],
                   "global_index": [[lib.ref_global_limb_index(g, loc, G)
                                     for loc in range(lib.ref_n_local_limbs(g, G, total))]
                                    for g in range(G)]}
            cases.append(rec)
    offs = [{"args": [p, l, nl, d], "local": lib.ref_local_buf_offset(p, l, nl, d),
             "global": lib.ref_global_buf_offset(p, l, nl, d)}
            for p in (0, 1, 2) for l in (0, 3) for nl in (5, 35) for d in (8192, 65536)]
    return {"cases": cases, "offsets": offs,
            "source": "src/multi_gpu/partition/rns_partition.cuh:29-107 via oracle/_ref"}


def main():
    default = os.path.join(os.path.dirname(ROOT), "reference")
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REF_ROOT", default)
    with open(os.path.join(HERE, "prime_kat.json"), "w") as f:
        json.dump(prime_kat(ref), f, indent=1)
    with open(os.path.join(HERE, "partition_ref.json"), "w") as f:
        json.dump(partition_ref(), f)
    print("wrote prime_kat.json, partition_ref.json")


if __name__ == "__main__":
    main()
