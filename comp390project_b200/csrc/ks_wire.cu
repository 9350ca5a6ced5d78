// ks_wire.cu -- byte format of evaluation keys and ciphertexts (host code).
//
// The reference has no serialised form: its key distribution is a stub that
// regenerates the keys on every GPU (distributed_context.cu:112-134).  Here a
// key or ciphertext is a self-describing little-endian blob that any rank can
// read from a file or a message and upload (each context keeps its shard):
//
//   offset size
//     0     8   magic "KSB2WIRE"
//     8     4   format version (2)
//    12     4   object: KS_WIRE_RELIN_KEY, KS_WIRE_GALOIS_KEY, KS_WIRE_CIPHERTEXT
//    16     4   Galois element (Galois keys: odd, < 2N), else 0
//    20     4   log_n
//    24     4   n_q (L)
//    28     4   n_p (alpha)
//    32     4   dim0: key digits ceil(L / alpha) | ciphertext polys
//    36     4   dim1: 2 | ciphertext level_limbs
//    40     4   dim2: L + alpha | 0
//    44     4   0 (reserved)
//    48     8   parameter digest: FNV-1a 64 of (log_n, q_0..q_{L-1}, p_0..p_{alpha-1})
//    56     8   blob digest: FNV-1a 64 of header bytes 0..55, then the payload bytes
//    64     -   payload: uint64 words in the in-memory layout
//                ([digits][2][L+alpha][N] keys, [polys][level_limbs][N] ciphertexts)
//
// Unpacking checks the magic, version, parameters, sizes, the Galois element,
// both digests (so a change to any header or payload byte is caught) and that
// every word is a canonical residue of its limb's prime.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/ks_capi.h"

namespace {

constexpr char kMagic[8] = {'K', 'S', 'B', '2', 'W', 'I', 'R', 'E'};
constexpr uint32_t kVersion = 2;
constexpr size_t kHeader = 64;

uint64_t fnv1a(uint64_t h, const void *data, size_t n) {
  const unsigned char *p = static_cast<const unsigned char *>(data);
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 0x100000001B3ull;
  }
  return h;
}
constexpr uint64_t kFnvBasis = 0xCBF29CE484222325ull;

uint64_t params_digest(const ks_params *prm) {
  uint64_t h = kFnvBasis;
  const uint64_t ln = prm->log_n;
  h = fnv1a(h, &ln, 8);
  for (int i = 0; i < prm->n_q; ++i) h = fnv1a(h, &prm->q[i], 8);
  for (int i = 0; i < prm->n_p; ++i) h = fnv1a(h, &prm->p[i], 8);
  return h;
}

struct Shape {
  uint32_t d0, d1, d2;
  size_t words;
};

// Words of the object and its dimensions; empty words on bad arguments.
Shape shape_of(const ks_params *prm, int object, int level_limbs, int n_polys) {
  const size_t N = (size_t)1 << prm->log_n;
  if (object == KS_WIRE_RELIN_KEY || object == KS_WIRE_GALOIS_KEY) {
    if (prm->n_p <= 0) return {0, 0, 0, 0};
    const uint32_t beta = (uint32_t)((prm->n_q + prm->n_p - 1) / prm->n_p);
    const uint32_t K = (uint32_t)(prm->n_q + prm->n_p);
    return {beta, 2, K, (size_t)beta * 2 * K * N};
  }
  if (object == KS_WIRE_CIPHERTEXT) {
    if (level_limbs < 1 || level_limbs > prm->n_q || n_polys < 1 || n_polys > 16)
      return {0, 0, 0, 0};
    return {(uint32_t)n_polys, (uint32_t)level_limbs, 0, (size_t)n_polys * level_limbs * N};
  }
  return {0, 0, 0, 0};
}

// Prime of word w of the object (keys: limb index kj of the key basis;
// ciphertexts: limb j of the level).
uint64_t prime_of_word(const ks_params *prm, int object, const Shape &sh, size_t w) {
  const size_t N = (size_t)1 << prm->log_n;
  const size_t limb = w / N;
  if (object == KS_WIRE_CIPHERTEXT) {
    const size_t j = limb % sh.d1;
    return prm->q[j];
  }
  const size_t kj = limb % sh.d2;
  return kj < (size_t)prm->n_q ? prm->q[kj] : prm->p[kj - prm->n_q];
}

bool params_ok(const ks_params *prm) {
  return prm && prm->q && prm->n_q >= 1 && prm->n_p >= 0 && (prm->n_p == 0 || prm->p) &&
         prm->log_n >= 1 && prm->log_n <= 20;
}

template <class T>
void put(unsigned char *b, size_t off, T v) {
  std::memcpy(b + off, &v, sizeof(T));
}
template <class T>
T get(const unsigned char *b, size_t off) {
  T v;
  std::memcpy(&v, b + off, sizeof(T));
  return v;
}

}  // namespace

extern "C" {

size_t ks_wire_size(const ks_params *prm, int object, int level_limbs, int n_polys) {
  if (!params_ok(prm)) return 0;
  const Shape sh = shape_of(prm, object, level_limbs, n_polys);
  return sh.words ? kHeader + sh.words * 8 : 0;
}

int ks_wire_pack(const ks_params *prm, int object, uint32_t galois_elt, int level_limbs,
                 int n_polys, const uint64_t *words, void *out, size_t cap) {
  if (!params_ok(prm) || !words || !out) return KS_ERR_INVALID;
  const Shape sh = shape_of(prm, object, level_limbs, n_polys);
  if (!sh.words || cap < kHeader + sh.words * 8) return KS_ERR_INVALID;
  if (object == KS_WIRE_GALOIS_KEY &&
      (!(galois_elt & 1u) || galois_elt >= (2ull << prm->log_n)))
    return KS_ERR_INVALID;
  unsigned char *b = static_cast<unsigned char *>(out);
  std::memset(b, 0, kHeader);
  std::memcpy(b, kMagic, 8);
  put<uint32_t>(b, 8, kVersion);
  put<uint32_t>(b, 12, (uint32_t)object);
  put<uint32_t>(b, 16, object == KS_WIRE_GALOIS_KEY ? galois_elt : 0u);
  put<uint32_t>(b, 20, prm->log_n);
  put<uint32_t>(b, 24, (uint32_t)prm->n_q);
  put<uint32_t>(b, 28, (uint32_t)prm->n_p);
  put<uint32_t>(b, 32, sh.d0);
  put<uint32_t>(b, 36, sh.d1);
  put<uint32_t>(b, 40, sh.d2);
  put<uint64_t>(b, 48, params_digest(prm));
  std::memcpy(b + kHeader, words, sh.words * 8);
  put<uint64_t>(b, 56, fnv1a(fnv1a(kFnvBasis, b, 56), words, sh.words * 8));
  return KS_OK;
}

int ks_wire_unpack(const ks_params *prm, const void *blob, size_t n, int *object,
                   uint32_t *galois_elt, int *level_limbs, int *n_polys, uint64_t *words,
                   size_t cap_words) {
  if (!params_ok(prm) || !blob || n < kHeader) return KS_ERR_INVALID;
  const unsigned char *b = static_cast<const unsigned char *>(blob);
  if (std::memcmp(b, kMagic, 8) != 0 || get<uint32_t>(b, 8) != kVersion) return KS_ERR_INVALID;
  const int obj = (int)get<uint32_t>(b, 12);
  if (get<uint32_t>(b, 20) != prm->log_n || get<uint32_t>(b, 24) != (uint32_t)prm->n_q ||
      get<uint32_t>(b, 28) != (uint32_t)prm->n_p || get<uint64_t>(b, 48) != params_digest(prm))
    return KS_ERR_INVALID;  // another parameter set
  const int ql = obj == KS_WIRE_CIPHERTEXT ? (int)get<uint32_t>(b, 36) : 0;
  const int np = obj == KS_WIRE_CIPHERTEXT ? (int)get<uint32_t>(b, 32) : 0;
  const Shape sh = shape_of(prm, obj, ql, np);
  if (!sh.words || get<uint32_t>(b, 32) != sh.d0 || get<uint32_t>(b, 36) != sh.d1 ||
      get<uint32_t>(b, 40) != sh.d2 || n != kHeader + sh.words * 8)
    return KS_ERR_INVALID;
  const uint32_t elt = get<uint32_t>(b, 16);
  const uint64_t two_n = 2ull << prm->log_n;
  if (obj == KS_WIRE_GALOIS_KEY ? (!(elt & 1u) || elt >= two_n) : elt != 0)
    return KS_ERR_INVALID;
  if (get<uint32_t>(b, 44) != 0) return KS_ERR_INVALID;
  if (fnv1a(fnv1a(kFnvBasis, b, 56), b + kHeader, sh.words * 8) != get<uint64_t>(b, 56))
    return KS_ERR_INVALID;
  for (size_t w = 0; w < sh.words; ++w)
    if (get<uint64_t>(b, kHeader + w * 8) >= prime_of_word(prm, obj, sh, w)) return KS_ERR_INVALID;
  if (object) *object = obj;
  if (galois_elt) *galois_elt = elt;
  if (level_limbs) *level_limbs = ql;
  if (n_polys) *n_polys = np;
  if (words) {
    if (cap_words < sh.words) return KS_ERR_INVALID;
    std::memcpy(words, b + kHeader, sh.words * 8);
  }
  return KS_OK;
}

}  // extern "C"
