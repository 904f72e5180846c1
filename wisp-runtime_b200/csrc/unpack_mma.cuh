// Packed codes -> bf16 MMA operands.
//
// A thread owns one 32-code unit of a row (BITS 32-bit words).  The unit is turned into 16 bf16x2
// registers ("pairs") with one LOP3 each: (w >> s) & mask | 0x43004300.  0x4300 is bf16 128.0, whose
// 7 mantissa bits have unit spacing, so a BITS-bit code q placed at mantissa bit p reads exactly
// 128 + 2^p q.  Each pair holds one code in the low half and one in the high half; which code and
// which p is fixed per bit width by the tables below (a shift is shared by up to three pairs).
//
// The MMA then sees A = 128 + 2^p q.  The matching B operand is built from the activation v as
// v * 2^-p for the same code, so A*B = 128 v 2^-p + q v: the product the dequant needs plus a bias
// 128 * sum(B) that is subtracted per quantization group, exactly.
//
// Pair p of a unit feeds MMA (m16n8k16) number p/2 of the group's eight; even p is the
// (k = 2c, 2c+1) register, odd p the (k = 2c+8, 2c+9) register, c = lane % 4.
#pragma once
#include "common.cuh"

namespace wisp {

struct PairSpec {
  uint8_t word;    // first word of the (funnel) window
  uint8_t shift;   // right shift of the window
  uint8_t funnel;  // 1: window = (w[word+1]:w[word]) >> shift
  uint8_t lo, lo_p, hi, hi_p;  // codes (index in the unit) and their mantissa bit positions
};

template <int BITS>
struct PairTable;

// 4-bit: word i, shift 4j -> nibbles (8i+j, 8i+4+j) at p = 0
template <>
struct PairTable<4> {
  __host__ __device__ static constexpr PairSpec get(int p) {
    constexpr PairSpec P[16] = {
      {0, 0, 0, 0, 0, 4, 0},   {0, 4, 0, 1, 0, 5, 0},   {0, 8, 0, 2, 0, 6, 0},   {0, 12, 0, 3, 0, 7, 0},
      {1, 0, 0, 8, 0, 12, 0},  {1, 4, 0, 9, 0, 13, 0},  {1, 8, 0, 10, 0, 14, 0}, {1, 12, 0, 11, 0, 15, 0},
      {2, 0, 0, 16, 0, 20, 0}, {2, 4, 0, 17, 0, 21, 0}, {2, 8, 0, 18, 0, 22, 0}, {2, 12, 0, 19, 0, 23, 0},
      {3, 0, 0, 24, 0, 28, 0}, {3, 4, 0, 25, 0, 29, 0}, {3, 8, 0, 26, 0, 30, 0}, {3, 12, 0, 27, 0, 31, 0},
    };
    return P[p];
  }
};

// 2-bit: word i; shift 0 -> crumbs (16i+{0,1,2}, +8) at p = {0,2,4}; shift 6 -> 16i+{3,4,5}; shift 12 -> 16i+{6,7}
template <>
struct PairTable<2> {
  __host__ __device__ static constexpr PairSpec get(int p) {
    constexpr PairSpec P[16] = {
      {0, 0, 0, 0, 0, 8, 0},    {0, 0, 0, 1, 2, 9, 2},    {0, 0, 0, 2, 4, 10, 4},   {0, 6, 0, 3, 0, 11, 0},
      {0, 6, 0, 4, 2, 12, 2},   {0, 6, 0, 5, 4, 13, 4},   {0, 12, 0, 6, 0, 14, 0},  {0, 12, 0, 7, 2, 15, 2},
      {1, 0, 0, 16, 0, 24, 0},  {1, 0, 0, 17, 2, 25, 2},  {1, 0, 0, 18, 4, 26, 4},  {1, 6, 0, 19, 0, 27, 0},
      {1, 6, 0, 20, 2, 28, 2},  {1, 6, 0, 21, 4, 29, 4},  {1, 12, 0, 22, 0, 30, 0}, {1, 12, 0, 23, 2, 31, 2},
    };
    return P[p];
  }
};

// 3-bit: code j at bit 3j of the 96-bit unit.  Fifteen pairs come from single windows (found by a
// search that minimises shifts); the sixteenth pairs code 0 (word 0, p = 0) with code 21 (bits 63..65,
// window (w2:w1) >> 15, p = 0) and needs one extra LOP3 to merge the two windows (entry 15, funnel = 2).
template <>
struct PairTable<3> {
  __host__ __device__ static constexpr PairSpec get(int p) {
    constexpr PairSpec P[16] = {
      {0, 0, 0, 1, 3, 6, 2},     {0, 5, 1, 2, 1, 8, 3},     {0, 5, 1, 3, 4, 7, 0},     {0, 11, 1, 5, 4, 9, 0},
      {0, 11, 1, 4, 1, 10, 3},   {1, 0, 0, 12, 4, 17, 3},   {1, 0, 0, 11, 1, 16, 0},   {1, 3, 1, 13, 4, 18, 3},
      {1, 9, 1, 14, 1, 20, 3},   {1, 9, 1, 15, 4, 19, 0},   {2, 0, 0, 22, 2, 27, 1},   {2, 4, 0, 24, 4, 29, 3},
      {2, 4, 0, 23, 1, 28, 0},   {2, 10, 0, 25, 1, 31, 3},  {2, 10, 0, 26, 4, 30, 0},  {1, 15, 2, 0, 0, 21, 0},
    };
    return P[p];
  }
};

template <int BITS>
__device__ __forceinline__ uint32_t pair_window(const uint32_t (&w)[BITS], const PairSpec& s) {
  if (s.funnel == 1) return __funnelshift_r(w[s.word], w[s.word + 1], s.shift);
  if (s.funnel == 2) return __funnelshift_r(w[s.word], w[s.word + 1], s.shift);
  return w[s.word] >> s.shift;
}

// pair p of a unit -> one bf16x2 A register
template <int BITS>
__device__ __forceinline__ uint32_t unpack_pair(const uint32_t (&w)[BITS], int p) {
  constexpr uint32_t M = (1u << BITS) - 1u;
  const PairSpec s = PairTable<BITS>::get(p);
  if (s.funnel == 2) {
    // code `lo` from word 0 at p = lo_p, code `hi` from the funnel window: two sources, one extra op
    const uint32_t lo = (w[0] >> (BITS * s.lo - s.lo_p)) & (M << s.lo_p);
    const uint32_t hi = pair_window<BITS>(w, s) & (M << (16 + s.hi_p));
    return (lo | hi) | 0x43004300u;
  }
  const uint32_t mask = (M << s.lo_p) | (M << (16 + s.hi_p));
  return (pair_window<BITS>(w, s) & mask) | 0x43004300u;
}

// unit words -> 16 bf16x2 A registers (pair order)
template <int BITS>
__device__ __forceinline__ void unpack_pairs(const uint32_t (&w)[BITS], uint32_t (&a)[16]) {
#pragma unroll
  for (int p = 0; p < 16; ++p) a[p] = unpack_pair<BITS>(w, p);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return uint32_t(f32_to_bf16(lo)) | (uint32_t(f32_to_bf16(hi)) << 16);
}

// scale of code position p in B (exact power of two)
__device__ __forceinline__ float pow2_neg(int p) { return __uint_as_float(uint32_t(127 - p) << 23); }

// Build the 16 B pairs of one unit from its 32 activation values (natural order), and the exact sum
// of the B values (for the 128 bias).  hi/lo split: part 0 = bf16(v), part 1 = bf16(v - bf16(v)).
template <int BITS>
__device__ __forceinline__ void build_b_pairs(const float (&v)[32], int part, uint32_t (&b)[16], float& bsum) {
  float s = 0.0f;
#pragma unroll
  for (int p = 0; p < 16; ++p) {
    const PairSpec sp = PairTable<BITS>::get(p);
    float lo = v[sp.lo] * pow2_neg(sp.lo_p);
    float hi = v[sp.hi] * pow2_neg(sp.hi_p);
    if (part == 1) {
      lo = lo - bf16_to_f32(f32_to_bf16(lo));
      hi = hi - bf16_to_f32(f32_to_bf16(hi));
    }
    b[p] = pack_bf16x2(lo, hi);
    s += bf16_to_f32(uint16_t(b[p])) + bf16_to_f32(uint16_t(b[p] >> 16));
  }
  bsum = s;
}

// D += A * B  (m16n8k16, bf16 inputs, fp32 accumulate)
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two 128-code groups of a 16-row MMA block (rows g and g+8 per lane), four independent accumulator
// chains.  wa*/wb*: the lane's unit words of rows g / g+8 for groups 0 and 1; b0/b1: the B pairs
// (zeros in lanes that hold no B column).  d0/d1 receive the two groups' results.
template <int BITS>
__device__ __forceinline__ void mma_two_groups(const uint32_t (&wa0)[BITS], const uint32_t (&wb0)[BITS],
                                               const uint32_t (&wa1)[BITS], const uint32_t (&wb1)[BITS],
                                               const uint32_t (&b0)[16], const uint32_t (&b1)[16], float (&d0)[4],
                                               float (&d1)[4]) {
  float e0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, e1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int i = 0; i < 4; ++i) d0[i] = d1[i] = 0.0f;
#pragma unroll
  for (int m = 0; m < 8; m += 2) {
    mma_bf16(d0, unpack_pair<BITS>(wa0, 2 * m), unpack_pair<BITS>(wb0, 2 * m), unpack_pair<BITS>(wa0, 2 * m + 1),
             unpack_pair<BITS>(wb0, 2 * m + 1), b0[2 * m], b0[2 * m + 1]);
    mma_bf16(d1, unpack_pair<BITS>(wa1, 2 * m), unpack_pair<BITS>(wb1, 2 * m), unpack_pair<BITS>(wa1, 2 * m + 1),
             unpack_pair<BITS>(wb1, 2 * m + 1), b1[2 * m], b1[2 * m + 1]);
    mma_bf16(e0, unpack_pair<BITS>(wa0, 2 * m + 2), unpack_pair<BITS>(wb0, 2 * m + 2),
             unpack_pair<BITS>(wa0, 2 * m + 3), unpack_pair<BITS>(wb0, 2 * m + 3), b0[2 * m + 2], b0[2 * m + 3]);
    mma_bf16(e1, unpack_pair<BITS>(wa1, 2 * m + 2), unpack_pair<BITS>(wb1, 2 * m + 2),
             unpack_pair<BITS>(wa1, 2 * m + 3), unpack_pair<BITS>(wb1, 2 * m + 3), b1[2 * m + 2], b1[2 * m + 3]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    d0[i] += e0[i];
    d1[i] += e1[i];
  }
}

}  // namespace wisp
