"""B200-native CKKS hybrid key switching (sm_100a CUDA behind a C ABI).

The product is libks_b200.so (include/ks_capi.h); this package is its Python
host side: the context wrapper, the reference-style key-switching entry
points, the cyclic limb partition, the wire format of keys and
ciphertexts, and the packing of the BSGS ciphertext x plaintext matmul.
"""
from .context import KsContext, KsGraph, gen_primes, nccl_unique_id, secret_generate  # noqa: F401
from ._capi import (KS_KEY_GALOIS, KS_KEY_RELIN, KS_MODE_INPUT_BROADCAST,  # noqa: F401
                    KS_MODE_OUTPUT_AGGREGATION, KsError)
from . import matmul, wire  # noqa: F401,E402
