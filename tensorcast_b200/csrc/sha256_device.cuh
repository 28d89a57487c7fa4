// SHA-256 (FIPS 180-4) building blocks for sm_100a device code.
//
// One 64-byte block is compressed entirely in registers: the 16-word message
// window rolls in place (fully unrolled, so every index is a compile-time
// constant), rotations are single funnel shifts (SHF.R.W), Ch and Maj are single
// three-input logic ops, and big-endian words come from __byte_perm.
// The round constants and initial hash value are the public constants of
// FIPS 180-4 sections 4.2.2 and 5.3.3.
#pragma once

#include <cstdint>

namespace tcx {
namespace dev {

static __constant__ uint32_t kRoundK[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

__device__ __forceinline__ void init_state(uint32_t s[8]) {
  s[0] = 0x6a09e667u; s[1] = 0xbb67ae85u; s[2] = 0x3c6ef372u; s[3] = 0xa54ff53au;
  s[4] = 0x510e527fu; s[5] = 0x9b05688cu; s[6] = 0x1f83d9abu; s[7] = 0x5be0cd19u;
}

__device__ __forceinline__ uint32_t rotr(uint32_t x, uint32_t n) { return __funnelshift_r(x, x, n); }
__device__ __forceinline__ uint32_t bswap32(uint32_t x) { return __byte_perm(x, 0u, 0x0123u); }
__device__ __forceinline__ uint32_t big_sigma0(uint32_t a) { return rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22); }
__device__ __forceinline__ uint32_t big_sigma1(uint32_t e) { return rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25); }
__device__ __forceinline__ uint32_t small_sigma0(uint32_t x) { return rotr(x, 7) ^ rotr(x, 18) ^ (x >> 3); }
__device__ __forceinline__ uint32_t small_sigma1(uint32_t x) { return rotr(x, 17) ^ rotr(x, 19) ^ (x >> 10); }
__device__ __forceinline__ uint32_t choose(uint32_t e, uint32_t f, uint32_t g) { return g ^ (e & (f ^ g)); }
__device__ __forceinline__ uint32_t majority(uint32_t a, uint32_t b, uint32_t c) { return (a & b) | (c & (a | b)); }

// Compresses one block whose 16 big-endian message words are in w (w is consumed).
__device__ __forceinline__ void compress(uint32_t s[8], uint32_t w[16]) {
  uint32_t a = s[0], b = s[1], c = s[2], d = s[3], e = s[4], f = s[5], g = s[6], h = s[7];
#pragma unroll
  for (int t = 0; t < 64; ++t) {
    if (t >= 16) {
      w[t & 15] += small_sigma1(w[(t - 2) & 15]) + w[(t - 7) & 15] + small_sigma0(w[(t - 15) & 15]);
    }
    const uint32_t t1 = h + big_sigma1(e) + choose(e, f, g) + kRoundK[t] + w[t & 15];
    const uint32_t t2 = big_sigma0(a) + majority(a, b, c);
    h = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + t2;
  }
  s[0] += a; s[1] += b; s[2] += c; s[3] += d;
  s[4] += e; s[5] += f; s[6] += g; s[7] += h;
}

// Read-only 16-byte load that bypasses L1 allocation (each block is read once).
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Big-endian words of a 64-byte block held as four 16-byte vectors.
__device__ __forceinline__ void words_from_vec(uint32_t w[16], const uint4& v0, const uint4& v1, const uint4& v2,
                                               const uint4& v3) {
  w[0] = bswap32(v0.x); w[1] = bswap32(v0.y); w[2] = bswap32(v0.z); w[3] = bswap32(v0.w);
  w[4] = bswap32(v1.x); w[5] = bswap32(v1.y); w[6] = bswap32(v1.z); w[7] = bswap32(v1.w);
  w[8] = bswap32(v2.x); w[9] = bswap32(v2.y); w[10] = bswap32(v2.z); w[11] = bswap32(v2.w);
  w[12] = bswap32(v3.x); w[13] = bswap32(v3.y); w[14] = bswap32(v3.z); w[15] = bswap32(v3.w);
}

// Writes the 32-byte big-endian digest of state s to a 16-byte aligned address.
__device__ __forceinline__ void store_digest(uint8_t* out, const uint32_t s[8]) {
  uint4* o = reinterpret_cast<uint4*>(out);
  o[0] = make_uint4(bswap32(s[0]), bswap32(s[1]), bswap32(s[2]), bswap32(s[3]));
  o[1] = make_uint4(bswap32(s[4]), bswap32(s[5]), bswap32(s[6]), bswap32(s[7]));
}

// Final block(s) of a message of msg_len bytes whose last rem (< 64) bytes start at tail:
// the tail bytes, 0x80, zero fill and the 64-bit big-endian bit length.
__device__ __forceinline__ void finish(uint32_t s[8], const uint8_t* tail, uint32_t rem, uint64_t msg_len) {
  uint32_t w[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t pos = 4u * k + j;
      uint32_t byte = 0;
      if (pos < rem) {
        byte = tail[pos];
      } else if (pos == rem) {
        byte = 0x80u;
      }
      word |= byte << (24 - 8 * j);
    }
    w[k] = word;
  }
  const uint64_t bits = msg_len * 8ull;
  if (rem < 56) {
    w[14] = static_cast<uint32_t>(bits >> 32);
    w[15] = static_cast<uint32_t>(bits);
    compress(s, w);
  } else {
    compress(s, w);
#pragma unroll
    for (int k = 0; k < 14; ++k) w[k] = 0;
    w[14] = static_cast<uint32_t>(bits >> 32);
    w[15] = static_cast<uint32_t>(bits);
    compress(s, w);
  }
}

}  // namespace dev
}  // namespace tcx
