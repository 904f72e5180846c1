// Packed codes -> u8 operands of the integer MMA (mma.sync m16n8k32, u8 x s8 -> s32).
//
// A lane owns one 32-code unit of a row (BITS 32-bit words) and turns it into 8 registers of 4 byte
// lanes each.  A byte lane holds one code q shifted left by p (the code sits wherever it already is
// inside the byte, p <= 5), so the lane's u8 value is exactly 2^p q and most registers are a single
// AND of a code word with a mask:
//   4-bit  w & 0x0F0F0F0F (p = 0) and w & 0xF0F0F0F0 (p = 4)                 8 ops per 32 codes
//   2-bit  w & (0x03030303 << 2t), t = 0..3 (p = 2t)                         8 ops per 32 codes
//   3-bit  the 24 codes that lie inside byte lanes of the three words: six ANDs; the 8 codes that
//          straddle bytes come from three shifted windows merged in two registers   13 ops per 32 codes
// The activation v of the same k-slot enters B as the integer limbs of round(v 2^(e - p)), so the
// slot contributes q v 2^e exactly up to that rounding; e is a per-128-code-group exponent that puts
// the group's largest |v| just below 2^22.  Three balanced base-256 limbs (B columns 0, 1, 2 =
// 2^16, 2^8, 1) carry 23 bits; every partial sum is an exact int32.
//
// Fragment use (m16n8k32): IMMA m of a group takes registers 2m (k = 4c..4c+3) and 2m+1
// (k = 16+4c..16+4c+3) of the lane's unit for row g (a0, a2) and row g+8 (a1, a3).
#pragma once
#include "common.cuh"

namespace wisp {

struct ByteTerm {
  uint8_t word, shift, funnel;  // window = funnel ? (w[word+1]:w[word]) >> shift : w[word] >> shift
  uint32_t mask;
};
struct ByteReg {
  uint8_t nterms;
  ByteTerm t[2];
  uint8_t code[4], p[4];  // byte lane b holds code[b] << p[b]
};

__host__ __device__ constexpr uint32_t m3(int a, int b = -1, int c = -1, int d = -1) {
  return (7u << a) | (b >= 0 ? 7u << b : 0u) | (c >= 0 ? 7u << c : 0u) | (d >= 0 ? 7u << d : 0u);
}

template <int BITS>
struct ByteTable;

template <>
struct ByteTable<4> {
  __host__ __device__ static constexpr ByteReg get(int r) {
    // r = 2i + h: word i, low (h = 0) or high (h = 1) nibbles; byte b holds code 8i + 2b + h
    return ByteReg{1,
                   {{uint8_t(r >> 1), 0, 0, (r & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu}, {0, 0, 0, 0u}},
                   {uint8_t(8 * (r >> 1) + (r & 1)), uint8_t(8 * (r >> 1) + 2 + (r & 1)),
                    uint8_t(8 * (r >> 1) + 4 + (r & 1)), uint8_t(8 * (r >> 1) + 6 + (r & 1))},
                   {uint8_t(4 * (r & 1)), uint8_t(4 * (r & 1)), uint8_t(4 * (r & 1)), uint8_t(4 * (r & 1))}};
  }
};

template <>
struct ByteTable<2> {
  __host__ __device__ static constexpr ByteReg get(int r) {
    // r = 4i + t: word i, crumb t of each byte; byte b holds code 16i + 4b + t at p = 2t
    return ByteReg{1,
                   {{uint8_t(r >> 2), 0, 0, 0x03030303u << (2 * (r & 3))}, {0, 0, 0, 0u}},
                   {uint8_t(16 * (r >> 2) + (r & 3)), uint8_t(16 * (r >> 2) + 4 + (r & 3)),
                    uint8_t(16 * (r >> 2) + 8 + (r & 3)), uint8_t(16 * (r >> 2) + 12 + (r & 3))},
                   {uint8_t(2 * (r & 3)), uint8_t(2 * (r & 3)), uint8_t(2 * (r & 3)), uint8_t(2 * (r & 3))}};
  }
};

template <>
struct ByteTable<3> {
  __host__ __device__ static constexpr ByteReg get(int r) {
    constexpr ByteReg R[8] = {
        {1, {{0, 0, 0, m3(0, 9, 18, 24)}, {0, 0, 0, 0u}}, {0, 3, 6, 8}, {0, 1, 2, 0}},
        {1, {{0, 0, 0, m3(3, 12, 21, 27)}, {0, 0, 0, 0u}}, {1, 4, 7, 9}, {3, 4, 5, 3}},
        {1, {{1, 0, 0, m3(1, 10, 16, 25)}, {0, 0, 0, 0u}}, {11, 14, 16, 19}, {1, 2, 0, 1}},
        {1, {{1, 0, 0, m3(4, 13, 19, 28)}, {0, 0, 0, 0u}}, {12, 15, 17, 20}, {4, 5, 3, 4}},
        {1, {{2, 0, 0, m3(2, 8, 17, 26)}, {0, 0, 0, 0u}}, {22, 24, 27, 30}, {2, 0, 1, 2}},
        {1, {{2, 0, 0, m3(5, 11, 20, 29)}, {0, 0, 0, 0u}}, {23, 25, 28, 31}, {5, 3, 4, 5}},
        // straddlers: (w1:w0) >> 2 gives codes 2, 5, 10; w2 >> 2 gives code 29
        {2, {{0, 2, 1, m3(4, 13, 28)}, {2, 2, 0, m3(21)}}, {2, 5, 29, 10}, {4, 5, 5, 4}},
        // (w2:w1) >> 4 gives codes 13, 18, 21; w2 >> 2 gives code 26
        {2, {{1, 4, 1, m3(3, 18, 27)}, {2, 2, 0, m3(12)}}, {13, 26, 18, 21}, {3, 4, 2, 3}},
    };
    return R[r];
  }
};

template <int BITS>
__device__ __forceinline__ uint32_t byte_window(const uint32_t (&w)[BITS], const ByteTerm& t) {
  if (t.funnel) return __funnelshift_r(w[t.word], w[t.word + 1], t.shift);
  return w[t.word] >> t.shift;
}

template <int BITS>
__device__ __forceinline__ uint32_t unpack_reg(const uint32_t (&w)[BITS], int r) {
  const ByteReg R = ByteTable<BITS>::get(r);
  uint32_t v = byte_window<BITS>(w, R.t[0]) & R.t[0].mask;
  if (R.nterms == 2) v |= byte_window<BITS>(w, R.t[1]) & R.t[1].mask;
  return v;
}

// exact int -> float for |i| < 2^22 without the conversion pipe
__device__ __forceinline__ float small_i2f(int i) { return __int_as_float(0x4B400000 + i) - 12582912.0f; }
// round-to-nearest-even float -> int for |f| < 2^22 without the conversion pipe
__device__ __forceinline__ int small_f2i(float f) { return __float_as_int(f + 12582912.0f) - 0x4B400000; }

// exponent e of a group with largest magnitude amax: amax * 2^e < 2^22 (e clamped to a normal float)
__device__ __forceinline__ int group_exponent(float amax) {
  const int E = int((__float_as_uint(amax) >> 23) & 0xFF);  // biased exponent: amax < 2^(E-126)
  int e = 148 - E;
  return e > 126 ? 126 : (e < -126 ? -126 : e);
}
__device__ __forceinline__ float pow2(int e) { return __uint_as_float(uint32_t(e + 127) << 23); }

// B limbs of one unit: L[limb][r] for the 8 registers (limb 0 = 2^16, 1 = 2^8, 2 = 1).
// For |xs| < 2^22 the balanced base-256 digits of xs (each in [-128, 127]) are exactly the bytes of
// (xs + 0x808080) ^ 0x808080 read as int8: adding 128 to every digit makes the digits of a 24-bit
// unsigned number, and XOR 0x80 turns a digit d + 128 back into the two's-complement byte of d.
// The magic-number rounding yields 0x4B400000 + xs, so one IADD and one XOR give all three limbs.
template <int BITS>
__device__ __forceinline__ void build_b_limbs(const float (&v)[32], int e, uint32_t (&L)[3][8]) {
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const ByteReg R = ByteTable<BITS>::get(r);
    uint32_t y[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const float f = v[R.code[b]] * pow2(e - R.p[b]) + 12582912.0f;  // round to nearest even
      y[b] = (__float_as_uint(f) + (0x808080u - 0x4B400000u)) ^ 0x808080u;
    }
    // gather byte l of y0..y3 into limb register l
    const uint32_t p01 = __byte_perm(y[0], y[1], 0x5140);  // y0.b0 y1.b0 y0.b1 y1.b1
    const uint32_t p23 = __byte_perm(y[2], y[3], 0x5140);
    const uint32_t q01 = __byte_perm(y[0], y[1], 0x0062);  // y0.b2 y1.b2 . .
    const uint32_t q23 = __byte_perm(y[2], y[3], 0x6200);  // . . y2.b2 y3.b2
    L[2][r] = __byte_perm(p01, p23, 0x5410);               // lo limbs
    L[1][r] = __byte_perm(p01, p23, 0x7632);               // mid limbs
    L[0][r] = __byte_perm(q01, q23, 0x7610);               // hi limbs
  }
}

// D += A * B  (m16n8k32, u8 A, s8 B, s32 accumulate)
__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 128-code group of a 16-row block: the lane's unit words of rows g (wa) and g+8 (wb), its B limb
// registers b (zeros in lanes that hold no limb column).  Two accumulator chains.
template <int BITS>
__device__ __forceinline__ void imma_group(const uint32_t (&wa)[BITS], const uint32_t (&wb)[BITS], const uint32_t (&b)[8],
                                           int (&d)[4]) {
  int e[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = 0;
  imma(d, unpack_reg<BITS>(wa, 0), unpack_reg<BITS>(wb, 0), unpack_reg<BITS>(wa, 1), unpack_reg<BITS>(wb, 1), b[0], b[1]);
  imma(e, unpack_reg<BITS>(wa, 2), unpack_reg<BITS>(wb, 2), unpack_reg<BITS>(wa, 3), unpack_reg<BITS>(wb, 3), b[2], b[3]);
  imma(d, unpack_reg<BITS>(wa, 4), unpack_reg<BITS>(wb, 4), unpack_reg<BITS>(wa, 5), unpack_reg<BITS>(wb, 5), b[4], b[5]);
  imma(e, unpack_reg<BITS>(wa, 6), unpack_reg<BITS>(wb, 6), unpack_reg<BITS>(wa, 7), unpack_reg<BITS>(wb, 7), b[6], b[7]);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] += e[i];
}

// Dot product of one 16-row block row per lane, from the limb columns (cols 0/1 in lane (g,0), col 2
// in lane (g,1)): lane c = 0 gets row g, lane c = 1 gets row g+8, both in the same instructions.
__device__ __forceinline__ float quad_row_dot(const int (&d)[4], int c) {
  const int x = __shfl_xor_sync(0xffffffffu, d[0], 1);  // c=0: row g col 2
  const int y = __shfl_xor_sync(0xffffffffu, d[2], 1);  // c=1: row g+8 col 0
  const int z = __shfl_xor_sync(0xffffffffu, d[3], 1);  // c=1: row g+8 col 1
  const int c0 = c == 0 ? d[0] : y, c1 = c == 0 ? d[1] : z, c2 = c == 0 ? x : d[2];
  return (small_i2f(c0) * 65536.0f + small_i2f(c1) * 256.0f) + small_i2f(c2);
}

}  // namespace wisp
