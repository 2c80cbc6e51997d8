// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The fp32 -> three-bf16 split of the tensor-core kernels and the no-swizzle K-major operand
// layout they store the parts in (shared memory) or hand to tcgen05.st (TMEM A operands).
//
// Split: x = x0 + x1 + x2, each part the round-to-nearest bf16 of what the previous ones leave;
// the two subtractions are exact, and what the three parts miss is below 2^-24 relative.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace cfa {
namespace tc {

// Byte offset of the 16-byte core-matrix row holding elements (row, 8 kc .. 8 kc + 7) of a K-major
// bf16 operand with 64 elements per row: core matrices of 8 rows x 16 bytes, K-adjacent core
// matrices 128 bytes apart, row groups of 8 rows 1024 bytes apart (desc_kmajor with LBO 128,
// SBO 1024).
__device__ __forceinline__ uint32_t kmaj_off(int row, int kc) {
  return static_cast<uint32_t>((((row >> 3) * 8 + kc) << 7) + ((row & 7) << 4));
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}

// Packed fp32 pairs (a 64-bit register pair, the first value low) and the sm_100 packed
// arithmetic on them: one instruction per pair where a scalar form takes two.
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// The round-to-nearest bf16 pair of a float pair (the low value in the low half).
__device__ __forceinline__ uint32_t to_bf2(uint64_t v) {
  float lo, hi;
  unpack2(v, lo, hi);
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
// The float pair a bf16 pair stands for (exact: a bf16 is the high half of its float).
__device__ __forceinline__ uint64_t from_bf2(uint32_t h) {
  return pack2(__uint_as_float(h << 16), __uint_as_float(h & 0xffff0000u));
}

// x[0..7] -> three 16-byte rows of bf16 parts (packed pairs, the even element low). Per pair:
// x0 = RN(x), x1 = RN(x - x0), x2 = RN(x - x0 - x1); both subtractions are exact.
__device__ __forceinline__ void split8(const float (&x)[8], uint4& p0, uint4& p1, uint4& p2) {
  uint32_t a[4], b[4], c[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t v = pack2(x[2 * i], x[2 * i + 1]);
    a[i] = to_bf2(v);
    const uint64_t r = sub2(v, from_bf2(a[i]));
    b[i] = to_bf2(r);
    c[i] = to_bf2(sub2(r, from_bf2(b[i])));
  }
  p0 = make_uint4(a[0], a[1], a[2], a[3]);
  p1 = make_uint4(b[0], b[1], b[2], b[3]);
  p2 = make_uint4(c[0], c[1], c[2], c[3]);
}

// x[0..15] -> the three parts of one K-step of 16 elements as 8 packed words each: a TMEM A
// operand's 8 columns (lane = row).
__device__ __forceinline__ void split16(const float (&x)[16], uint32_t (&p)[3][8]) {
  float lo[8], hi[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    lo[u] = x[u];
    hi[u] = x[8 + u];
  }
  uint4 l[3], h[3];
  split8(lo, l[0], l[1], l[2]);
  split8(hi, h[0], h[1], h[2]);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    p[i][0] = l[i].x, p[i][1] = l[i].y, p[i][2] = l[i].z, p[i][3] = l[i].w;
    p[i][4] = h[i].x, p[i][5] = h[i].y, p[i][6] = h[i].z, p[i][7] = h[i].w;
  }
}

// The parts of x[0..7] into three part buffers `part_bytes` apart, at byte offset `off`.
__device__ __forceinline__ void store_parts(unsigned char* base, int part_bytes, uint32_t off,
                                            const float (&x)[8]) {
  uint4 p0, p1, p2;
  split8(x, p0, p1, p2);
  *reinterpret_cast<uint4*>(base + off) = p0;
  *reinterpret_cast<uint4*>(base + part_bytes + off) = p1;
  *reinterpret_cast<uint4*>(base + 2 * part_bytes + off) = p2;
}

// 8 consecutive 32-bit TMEM columns of this thread's lane (32x32b shape), store / load.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}

// 4 consecutive 32-bit TMEM columns of this thread's lane (32x32b shape), store.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint4& v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace tc
}  // namespace cfa
