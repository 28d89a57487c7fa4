/*
 * tcx_oracle.c -- CPU ORACLE. TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker for the GPU content-hashing path, never the thing
 * measured or shipped. Only tests/, __graft_entry__.smoke() and the CPU legs of
 * bench.py load it. The product library (tensorcast_b200/csrc) never links it.
 *
 * It restates, in plain C, the reference's CPU hashing path:
 *   - sha256_bytes            core/common/artifact_hash_cpu.cc:161-196
 *                             (an empty span yields 32 zero bytes, not SHA-256(""))
 *   - compute_tree_hash_sha256  artifact_hash_cpu.cc:198-233
 *                             (pairwise; an odd trailing node is promoted unchanged)
 *   - base32_lower_encode     artifact_hash_cpu.cc:33-64
 *   - to_multibase_multihash_sha256  artifact_hash_cpu.cc:235-254 ('b' + base32(0x12 0x20 || digest))
 *   - compute_chunk_lengths   artifact_hash_cpu.cc:256-267
 *   - determine_leaf_chunk_size  artifact_hash_cpu.cc:269-303 (+ constants artifact_hash_internal.h:15-17,
 *                             artifact_hash.h:16)
 *   - compute_data_multihash_from_seekable_source  source_hash.cc:19-61 (leaf size used as given)
 *
 * The reference computes SHA-256 through OpenSSL EVP_sha256 (system libcrypto 3.x;
 * artifact_hash_cpu.cc:14-15,161-196). SHA-256 itself is the published FIPS 180-4
 * algorithm; it is restated here from the standard (section 6.2), and the test suite
 * pins this restatement against the NIST example vectors, Python hashlib and the
 * reference's own golden view-id vector. A second leaf-digest entry point calls
 * OpenSSL EVP exactly as the reference does; it serves as the timed CPU baseline.
 */
#include <openssl/evp.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define TCXO_OK 0
#define TCXO_INVALID_ARGUMENT 3
#define TCXO_INTERNAL 13

/* FIPS 180-4 section 4.2.2: first 32 bits of the fractional parts of the cube roots
 * of the first 64 primes. */
static const uint32_t K256[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

/* FIPS 180-4 section 5.3.3: initial hash value. */
static const uint32_t H0[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                               0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};

static inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static void compress(uint32_t st[8], const uint8_t blk[64]) {
  uint32_t w[64];
  for (int t = 0; t < 16; ++t) {
    w[t] = ((uint32_t)blk[4 * t] << 24) | ((uint32_t)blk[4 * t + 1] << 16) | ((uint32_t)blk[4 * t + 2] << 8) |
           (uint32_t)blk[4 * t + 3];
  }
  for (int t = 16; t < 64; ++t) {
    uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
    uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
    w[t] = s1 + w[t - 7] + s0 + w[t - 16];
  }
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
  for (int t = 0; t < 64; ++t) {
    uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    uint32_t ch = (e & f) ^ (~e & g);
    uint32_t t1 = h + S1 + ch + K256[t] + w[t];
    uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
    uint32_t t2 = S0 + mj;
    h = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + t2;
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d;
  st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

/* Plain FIPS 180-4 SHA-256 of len bytes (len may be 0: SHA-256 of the empty message). */
void tcxo_sha256(const uint8_t* data, uint64_t len, uint8_t out[32]) {
  uint32_t st[8];
  memcpy(st, H0, sizeof st);
  uint64_t full = len / 64;
  for (uint64_t i = 0; i < full; ++i) compress(st, data + 64 * i);
  uint8_t tail[128];
  uint64_t rem = len - full * 64;
  memset(tail, 0, sizeof tail);
  if (rem) memcpy(tail, data + full * 64, (size_t)rem);
  tail[rem] = 0x80;
  int nblk = rem < 56 ? 1 : 2;
  uint64_t bits = len * 8u;
  for (int i = 0; i < 8; ++i) tail[nblk * 64 - 1 - i] = (uint8_t)(bits >> (8 * i));
  compress(st, tail);
  if (nblk == 2) compress(st, tail + 64);
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = (uint8_t)(st[i] >> 24);
    out[4 * i + 1] = (uint8_t)(st[i] >> 16);
    out[4 * i + 2] = (uint8_t)(st[i] >> 8);
    out[4 * i + 3] = (uint8_t)st[i];
  }
}

/* artifact_hash_cpu.cc:161-164: the reference returns 32 zero bytes for an empty span. */
void tcxo_sha256_bytes(const uint8_t* data, uint64_t len, uint8_t out[32]) {
  if (len == 0) {
    memset(out, 0, 32);
    return;
  }
  tcxo_sha256(data, len, out);
}

/* OpenSSL EVP_sha256, called the way artifact_hash_cpu.cc:166-195 calls it. */
int tcxo_sha256_openssl(const uint8_t* data, uint64_t len, uint8_t out[32]) {
  if (len == 0) {
    memset(out, 0, 32);
    return TCXO_OK;
  }
  EVP_MD_CTX* ctx = EVP_MD_CTX_new();
  if (!ctx) return TCXO_INTERNAL;
  unsigned int out_len = 0;
  int ok = EVP_DigestInit_ex(ctx, EVP_sha256(), NULL) == 1 && EVP_DigestUpdate(ctx, data, (size_t)len) == 1 &&
           EVP_DigestFinal_ex(ctx, out, &out_len) == 1 && out_len == 32;
  EVP_MD_CTX_free(ctx);
  return ok ? TCXO_OK : TCXO_INTERNAL;
}

/* artifact_hash_cpu.cc:256-267 / source_hash.cc:32: number of leaves of size <= leaf. */
uint64_t tcxo_leaf_count(uint64_t total, uint64_t leaf) {
  if (leaf == 0) return 0;
  return (total + leaf - 1) / leaf;
}

/* source_hash.cc:38-58: leaves [i*L, min((i+1)*L, T)) hashed in order, one digest each.
 * out must hold tcxo_leaf_count(total, leaf) * 32 bytes. */
int tcxo_leaf_digests(const uint8_t* buf, uint64_t total, uint64_t leaf, uint8_t* out) {
  if (total == 0 || leaf == 0) return TCXO_INVALID_ARGUMENT;
  uint64_t n = tcxo_leaf_count(total, leaf);
  for (uint64_t i = 0; i < n; ++i) {
    uint64_t off = i * leaf;
    uint64_t len = total - off < leaf ? total - off : leaf;
    tcxo_sha256_bytes(buf + off, len, out + 32 * i);
  }
  return TCXO_OK;
}

struct ossl_job {
  const uint8_t* buf;
  uint64_t total, leaf, first, last;
  uint8_t* out;
  int rc;
};

static void* ossl_worker(void* p) {
  struct ossl_job* j = (struct ossl_job*)p;
  j->rc = TCXO_OK;
  for (uint64_t i = j->first; i < j->last; ++i) {
    uint64_t off = i * j->leaf;
    uint64_t len = j->total - off < j->leaf ? j->total - off : j->leaf;
    int rc = tcxo_sha256_openssl(j->buf + off, len, j->out + 32 * i);
    if (rc != TCXO_OK) j->rc = rc;
  }
  return NULL;
}

/* Same leaves as tcxo_leaf_digests, hashed by OpenSSL. threads <= 1 runs the reference's
 * single-threaded loop (source_hash.cc:38-58); threads > 1 splits the leaf range. */
int tcxo_leaf_digests_openssl(const uint8_t* buf, uint64_t total, uint64_t leaf, uint8_t* out, int threads) {
  if (total == 0 || leaf == 0) return TCXO_INVALID_ARGUMENT;
  uint64_t n = tcxo_leaf_count(total, leaf);
  if (threads <= 1 || n < 2) {
    struct ossl_job j = {buf, total, leaf, 0, n, out, 0};
    ossl_worker(&j);
    return j.rc;
  }
  if ((uint64_t)threads > n) threads = (int)n;
  struct ossl_job* jobs = (struct ossl_job*)calloc((size_t)threads, sizeof *jobs);
  pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof *tids);
  if (!jobs || !tids) {
    free(jobs);
    free(tids);
    return TCXO_INTERNAL;
  }
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (struct ossl_job){buf, total, leaf, n * (uint64_t)t / (uint64_t)threads,
                                n * (uint64_t)(t + 1) / (uint64_t)threads, out, 0};
    pthread_create(&tids[t], NULL, ossl_worker, &jobs[t]);
  }
  int rc = TCXO_OK;
  for (int t = 0; t < threads; ++t) {
    pthread_join(tids[t], NULL);
    if (jobs[t].rc != TCXO_OK) rc = jobs[t].rc;
  }
  free(jobs);
  free(tids);
  return rc;
}

/* artifact_hash_cpu.cc:198-233. digests: n*32 bytes (not modified). */
int tcxo_tree_root(const uint8_t* digests, uint64_t n, uint8_t root[32]) {
  if (n == 0) return TCXO_INVALID_ARGUMENT;
  uint8_t* level = (uint8_t*)malloc((size_t)n * 32);
  if (!level) return TCXO_INTERNAL;
  memcpy(level, digests, (size_t)n * 32);
  uint64_t m = n;
  while (m > 1) {
    uint64_t next = 0;
    for (uint64_t i = 0; i < m; i += 2) {
      if (i + 1 < m) {
        uint8_t concat[64];
        memcpy(concat, level + 32 * i, 32);
        memcpy(concat + 32, level + 32 * (i + 1), 32);
        tcxo_sha256_bytes(concat, 64, level + 32 * next);
      } else {
        memmove(level + 32 * next, level + 32 * i, 32);
      }
      ++next;
    }
    m = next;
  }
  memcpy(root, level, 32);
  free(level);
  return TCXO_OK;
}

/* artifact_hash_cpu.cc:33-64 (RFC 4648 alphabet, lower case, no padding) and :235-254.
 * out receives 'b' + 55 base32 characters + NUL (57 bytes). */
int tcxo_multihash(const uint8_t digest[32], char* out, uint64_t cap) {
  static const char alpha[] = "abcdefghijklmnopqrstuvwxyz234567";
  uint8_t mh[34];
  mh[0] = 0x12;
  mh[1] = 0x20;
  memcpy(mh + 2, digest, 32);
  const uint64_t in_len = 34, out_len = (in_len * 8 + 4) / 5; /* 55 */
  if (cap < out_len + 2) return TCXO_INVALID_ARGUMENT;
  char tmp[72];
  uint64_t pos = 0;
  for (uint64_t i = 0; i < in_len;) {
    uint64_t take = in_len - i < 5 ? in_len - i : 5;
    uint64_t acc = 0;
    for (uint64_t j = 0; j < take; ++j) acc = (acc << 8) | mh[i + j];
    acc <<= (5 - take) * 8;
    for (int s = 35; s >= 0; s -= 5) tmp[pos++] = alpha[(acc >> s) & 31];
    i += take;
  }
  out[0] = 'b';
  memcpy(out + 1, tmp, (size_t)out_len);
  out[out_len + 1] = '\0';
  return TCXO_OK;
}

/* artifact_hash_cpu.cc:269-303 with kMaxChunkSize = 64 MiB, kMinLeafChunkBytes = 512 KiB,
 * kTargetLeafCount = 4096 (artifact_hash_internal.h:15-17) and the 4 MiB default
 * (artifact_hash.h:16). Only the exact default request triggers the halving policy. */
uint64_t tcxo_determine_leaf_chunk_size(uint64_t total, uint64_t requested) {
  const uint64_t kDefault = 4ull << 20, kMax = 64ull << 20, kMin = 512ull << 10, kTarget = 4096;
  uint64_t bounded = requested == 0 ? kDefault : requested;
  if (bounded > kMax) bounded = kMax;
  if (bounded < 64) bounded = 64;
  bounded -= bounded % 64;
  if (bounded == 0) bounded = 64;
  if (requested != kDefault) return bounded;
  uint64_t adjusted = bounded;
  while (adjusted > kMin && (total + adjusted - 1) / adjusted < kTarget) {
    uint64_t cand = adjusted / 2;
    cand -= cand % 64;
    if (cand < kMin) break;
    adjusted = cand;
  }
  if (adjusted < kMin) adjusted = kMin;
  return adjusted == 0 ? 64 : adjusted;
}

/* compute_data_multihash_from_cpu_memory (source_hash.cc:63-70 -> :19-61): the leaf size
 * is used exactly as given. out: 57 bytes. use_openssl selects the EVP leaf hasher. */
int tcxo_multihash_from_cpu_memory(const uint8_t* buf, uint64_t total, uint64_t leaf, char* out, uint64_t cap,
                                   int use_openssl, int threads) {
  if (total == 0 || leaf == 0) return TCXO_INVALID_ARGUMENT;
  uint64_t n = tcxo_leaf_count(total, leaf);
  uint8_t* d = (uint8_t*)malloc((size_t)n * 32);
  if (!d) return TCXO_INTERNAL;
  int rc = use_openssl ? tcxo_leaf_digests_openssl(buf, total, leaf, d, threads) : tcxo_leaf_digests(buf, total, leaf, d);
  uint8_t root[32];
  if (rc == TCXO_OK) rc = tcxo_tree_root(d, n, root);
  free(d);
  if (rc == TCXO_OK) rc = tcxo_multihash(root, out, cap);
  return rc;
}
