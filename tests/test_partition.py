"""Partition math against the reference's own code (rns_partition.cuh,
compiled under oracle/_ref when available, and its committed outputs)."""
import ctypes as C
import json
import os

import pytest

from comp390project_b200 import partition as P

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_partition.so")


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(ROOT, "tests", "golden", "partition_ref.json")) as f:
        return json.load(f)


def test_matches_reference_golden_outputs(golden):
    for rec in golden["cases"]:
        G, total = rec["G"], rec["total"]
        assert [P.owner_of_limb(j, G) for j in range(total)] == rec["owner"]
        assert [P.local_index_of_limb(j, G) for j in range(total)] == rec["local_index"]
        assert [P.n_local_limbs(g, G, total) for g in range(G)] == rec["n_local"]
        assert [[P.global_limb_index(g, loc, G) for loc in range(P.n_local_limbs(g, G, total))]
                for g in range(G)] == rec["global_index"]
        assert [P.limbs_for_gpu(g, G, total) for g in range(G)] == rec["global_index"]
    for rec in golden["offsets"]:
        p, l, nl, d = rec["args"]
        assert P.local_buf_offset(p, l, nl, d) == rec["local"]
        assert P.global_buf_offset(p, l, nl, d) == rec["global"]


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference partition library not built")
def test_matches_reference_library_live():
    lib = C.CDLL(REF_SO)
    sz = C.c_size_t
    lib.ref_n_local_limbs.restype = sz
    lib.ref_n_local_limbs.argtypes = [C.c_int, C.c_int, sz]
    lib.ref_limbs_for_gpu.restype = C.c_int
    lib.ref_limbs_for_gpu.argtypes = [C.c_int, C.c_int, sz, C.POINTER(sz), C.c_int]
    for G in range(1, 9):
        for total in range(0, 45):
            for g in range(G):
                assert lib.ref_n_local_limbs(g, G, total) == P.n_local_limbs(g, G, total)
                buf = (sz * 64)()
                n = lib.ref_limbs_for_gpu(g, G, total, buf, 64)
                assert list(buf[:n]) == P.limbs_for_gpu(g, G, total)


def test_gathered_slots_cover_every_limb_once():
    for G in (1, 2, 3, 4, 8):
        for total in (1, 5, 35, 40):
            ml = P.max_local(total, G)
            slots = [P.gathered_slot(j, G, total) for j in range(total)]
            assert len(set(slots)) == total and max(slots) < G * ml
            # slot order equals the rank-grouped order of a padded all-gather
            for j in range(total):
                g, loc = P.owner_of_limb(j, G), P.local_index_of_limb(j, G)
                assert P.gathered_slot(j, G, total) == g * ml + loc


def test_output_limbs_partition_the_extended_basis():
    L, alpha = 35, 5
    for G in (1, 2, 4, 8):
        for Ql in (35, 20, 1):
            outs = [P.owned_output_limbs(g, G, Ql, L, alpha) for g in range(G)]
            flat = sorted(x for o in outs for x in o)
            assert flat == list(range(Ql + alpha))
            keys = [P.owned_key_limbs(g, G, L, alpha) for g in range(G)]
            assert sorted(x for k in keys for x in k) == list(range(L + alpha))
        if Ql == 35 and G == 8:
            assert all(len(o) == 5 for o in outs)  # 40 limbs, 5 per rank
