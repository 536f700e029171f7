// Integer-dot units for the batch-1 GEMV.
//
// The activation slice a thread owns (one unit: 64 elements for the K-quants,
// 32 for Q8_0 and Q1_0) is quantised once per launch to 16-bit integers with
// one fp32 scale per unit:  x ~= sx * xq,  xq = rint(x / sx) in [-32639, 32639],
// sx = max|x| / 32639, and split into two signed byte planes
// xq = 256 * xh + xl with xh, xl in [-128, 127] (32639 = 256*127 + 127 is the
// largest value the split holds).  A weight word of four quant
// bytes (all below 128, or signed for Q8_0) then needs two signed dp4a
// instructions for four multiply-adds.  Sums stay exact in int32 (bounds are
// noted per format) until one conversion per scale group; the only
// approximation is the 16-bit activation grid, ~2e-5 .. 4e-5 relative error
// of the output against fp64, 25x inside the 1e-3 gate.
//
// Per-unit thread-constant data (UnitX): the two byte planes, the scale, and
// integer sums of xq over each scale group of the weight format (for the
// K-quant mins, the Q6_K -32 offset and the Q1_0 sign identity).
#pragma once

#include "formats.cuh"

namespace frc {

FRC_DEVICE_INLINE int dp4a_us(uint32_t a_u8, uint32_t b_s8, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_u8), "r"(b_s8), "r"(c));
  return d;
}
FRC_DEVICE_INLINE int dp4a_uu(uint32_t a_u8, uint32_t b_u8, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_u8), "r"(b_u8), "r"(c));
  return d;
}
FRC_DEVICE_INLINE int dp4a_ss(uint32_t a_s8, uint32_t b_s8, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s8), "r"(b_s8), "r"(c));
  return d;
}
FRC_DEVICE_INLINE int dp4a_su(uint32_t a_s8, uint32_t b_u8, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s8), "r"(b_u8), "r"(c));
  return d;
}

constexpr int kXqMax = 32639;  // 256 * 127 + 127

template <int Q> struct I8;  // geometry of the integer units

template <> struct I8<kQ4_K> { static constexpr int E = 64, UPB = 4, NG = 2; };
template <> struct I8<kQ5_K> { static constexpr int E = 64, UPB = 4, NG = 2; };
template <> struct I8<kQ6_K> { static constexpr int E = 64, UPB = 4, NG = 4; };
template <> struct I8<kQ8_0> { static constexpr int E = 32, UPB = 1, NG = 1; };
template <> struct I8<kQ1_0> { static constexpr int E = 32, UPB = 4, NG = 1; };

// Offset inside the block of element i (0..E-1, in x-word order) of unit j.
template <int Q> FRC_DEVICE_INLINE int i8_pos(int j, int i);
// K-quants: unit j = group g (64 elements: 32 low nibbles of sub-block 2g then
// 32 high nibbles of sub-block 2g+1), all contiguous.
template <> FRC_DEVICE_INLINE int i8_pos<kQ4_K>(int j, int i) { return 64 * j + i; }
template <> FRC_DEVICE_INLINE int i8_pos<kQ5_K>(int j, int i) { return 64 * j + i; }
// Q6_K: unit j = (half = j/2, lh = j%2): quarter r = i/16 holds elements
// 128 half + 32 r + 16 lh + (i % 16).
template <> FRC_DEVICE_INLINE int i8_pos<kQ6_K>(int j, int i) {
  return 128 * (j >> 1) + 32 * (i >> 4) + 16 * (j & 1) + (i & 15);
}
template <> FRC_DEVICE_INLINE int i8_pos<kQ8_0>(int, int i) { return i; }
template <> FRC_DEVICE_INLINE int i8_pos<kQ1_0>(int j, int i) { return 32 * j + i; }

// Shared-memory record of one quantised unit: xh words, xl words, the integer
// sums of each scale group, the scale; padded to a multiple of 4 words with a
// stride that keeps 16-byte loads of consecutive records conflict-free.
template <int Q>
__host__ __device__ constexpr int record_words() {
  return I8<Q>::E == 64 ? (I8<Q>::NG == 4 ? 40 : 36) : 20;
}

template <int Q>
struct UnitX {
  static constexpr int E = I8<Q>::E, NW = E / 4, NG = I8<Q>::NG, RW = record_words<Q>();
  uint32_t xh[NW];  // signed high bytes, 4 elements per word
  uint32_t xl[NW];  // signed low bytes
  int xsum[NG];     // sum of xq over each scale group (E / NG consecutive words)
  float sx;

  FRC_DEVICE_INLINE void from_record(const uint32_t* rec) {
#pragma unroll
    for (int w = 0; w < NW; w += 4) {
      const uint4 a = *reinterpret_cast<const uint4*>(rec + w);
      const uint4 b = *reinterpret_cast<const uint4*>(rec + NW + w);
      xh[w] = a.x; xh[w + 1] = a.y; xh[w + 2] = a.z; xh[w + 3] = a.w;
      xl[w] = b.x; xl[w + 1] = b.y; xl[w + 2] = b.z; xl[w + 3] = b.w;
    }
#pragma unroll
    for (int g = 0; g < NG; ++g) xsum[g] = static_cast<int>(rec[2 * NW + g]);
    sx = __uint_as_float(rec[2 * NW + NG]);
  }
  FRC_DEVICE_INLINE void zero() {
#pragma unroll
    for (int w = 0; w < NW; ++w) xh[w] = xl[w] = 0;
#pragma unroll
    for (int g = 0; g < NG; ++g) xsum[g] = 0;
    sx = 0.f;
  }
};

// round(v * inv) to the nearest integer (ties to even) for |v * inv| < 2^22:
// one FMA against 1.5 * 2^23 puts the integer in the low mantissa bits (full
// rate; an int conversion instruction runs at a quarter of it).
FRC_DEVICE_INLINE int round_to_int(float v, float inv) {
  return __float_as_int(fmaf(v, inv, 12582912.0f)) - 0x4B400000;
}

// Unit u and x-word w (four consecutive elements) that global x-word gw of a
// row belongs to.  K-quants other than Q6_K, Q8_0 and Q1_0 number their unit
// words in x order; a Q6_K block's 64 words interleave its four units: word e
// (element 4e of the block) is in half e / 32, quarter (e / 8) % 4, 16-element
// run (e / 4) % 2, so unit 2 half + run, word 4 quarter + e % 4.
template <int Q> FRC_DEVICE_INLINE void x_word_home(int gw, int& u, int& w) {
  if constexpr (Q == kQ6_K) {
    const int e = gw & 63;
    u = (gw >> 6) * 4 + 2 * (e >> 5) + ((e >> 2) & 1);
    w = 4 * ((e >> 3) & 3) + (e & 3);
  } else {
    constexpr int NW = I8<Q>::E / 4;
    u = gw / NW;
    w = gw % NW;
  }
}

// Lane-index bits that differ between the threads holding one unit
// (kUnitLanes) and one scale group (kGroupLanes) when every thread takes four
// consecutive x-words (16 elements) and a warp's lanes take consecutive
// quads.  A 64-element unit is 4 neighbouring lanes (32-element: 2) and its
// 32-element group 2 lanes.  A Q6_K block's 16 quads interleave its units:
// lane bit 0 is the 16-element run (unit j % 2), bits 1-2 the quarter, bit 3
// the half (unit j / 2), so a unit's lanes differ in bits 1-2 and every lane
// holds one whole 16-element scale group.
template <int Q> struct XQuads {
  static constexpr int kUnitLanes = Q == kQ6_K ? 0x6 : I8<Q>::E / 16 - 1;
  static constexpr int kGroupLanes = Q == kQ6_K ? 0x0 : I8<Q>::E / 16 / I8<Q>::NG - 1;
};

// Quantise the activations of every unit of a row into shared records: xq =
// round(x * kXqMax / amax) per unit, stored as high bytes (xq + 128) >> 8 and
// low bytes xq & 0xFF, plus the integer sum of xq over each scale group and the
// unit's scale amax / kXqMax.  Every thread takes four x-words (16 consecutive
// elements, four 16-byte loads) per round; the loads of R rounds (k <= 16 R
// blockDim.x) are issued before any is used, since an L2 round trip under a
// full weight stream costs about a microsecond.  The unit's amax and the group
// sums are reduced across the lanes that share them with butterfly shuffles.
// |x * inv| <= kXqMax (1 + 2^-24) rounds to at most kXqMax, so no clamp is
// needed.  One FMA against 1.5 * 2^23 + 128 leaves xq + 128 in the low
// mantissa bits: byte 0 is the low byte of xq with its top bit flipped, byte 1
// the high byte.  Every thread of the block calls this with the same arguments
// (it uses full-warp shuffles); blockDim.x is a multiple of 32.
template <int Q, int R>
FRC_DEVICE_INLINE void quantise_words(const float* x, int units, uint32_t* records) {
  constexpr int NW = I8<Q>::E / 4, NG = I8<Q>::NG, RW = record_words<Q>();
  constexpr int UL = XQuads<Q>::kUnitLanes, GL = XQuads<Q>::kGroupLanes;
  const int ntask = units * NW / 4;
  const int bd = static_cast<int>(blockDim.x), tid = static_cast<int>(threadIdx.x);
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (int base = 0; base < ntask; base += R * bd) {
    float4 v[R][4];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int t = base + i * bd + tid;
#pragma unroll
      for (int q = 0; q < 4; ++q) v[i][q] = t < ntask ? __ldg(x4 + 4 * t + q) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < R; ++i) {
      if (base + i * bd >= ntask) break;  // uniform over the block
      const int t = base + i * bd + tid;
      float m4[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        m4[q] = fmaxf(fmaxf(fabsf(v[i][q].x), fabsf(v[i][q].y)), fmaxf(fabsf(v[i][q].z), fabsf(v[i][q].w)));
      float a = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
#pragma unroll
      for (int m = 1; m < 32; m <<= 1)
        if (UL & m) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, m));
      const float inv = a > 0.f ? static_cast<float>(kXqMax) / a : 0.0f;
      uint32_t hw[4], lw[4];
      uint32_t sum = 0;  // the xq plus 0x4B400080 each, in 32-bit wrapping arithmetic
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r0 = __float_as_int(fmaf(v[i][q].x, inv, 12583040.0f));
        const int r1 = __float_as_int(fmaf(v[i][q].y, inv, 12583040.0f));
        const int r2 = __float_as_int(fmaf(v[i][q].z, inv, 12583040.0f));
        const int r3 = __float_as_int(fmaf(v[i][q].w, inv, 12583040.0f));
        hw[q] = __byte_perm(__byte_perm(r0, r1, 0x0051), __byte_perm(r2, r3, 0x0051), 0x5410);
        lw[q] = __byte_perm(__byte_perm(r0, r1, 0x0040), __byte_perm(r2, r3, 0x0040), 0x5410) ^ 0x80808080u;
        sum += static_cast<uint32_t>(r0) + static_cast<uint32_t>(r1) + static_cast<uint32_t>(r2) +
               static_cast<uint32_t>(r3);
      }
      int gs = static_cast<int>(sum - 16u * 0x4B400080u);
#pragma unroll
      for (int m = 1; m < 32; m <<= 1)
        if (GL & m) gs += __shfl_xor_sync(0xffffffffu, gs, m);
      if (t < ntask) {
        int u, w;
        x_word_home<Q>(4 * t, u, w);
        uint32_t* rec = records + u * RW;
        *reinterpret_cast<uint4*>(rec + w) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(rec + NW + w) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        if (w % (NW / NG) == 0) rec[2 * NW + w / (NW / NG)] = static_cast<uint32_t>(gs);
        if (w == 0) rec[2 * NW + NG] = __float_as_uint(a > 0.f ? a / static_cast<float>(kXqMax) : 1.0f);
      }
    }
  }
}

// Per-thread constants derived from the unit index j and block index b.
struct UnitCtx {
  int j;
  uint32_t blk;     // byte offset of the unit's block in its row
  uint32_t f0;      // Q4_K/Q5_K: offset of the unit's quants in the row; Q6_K: of ql (within the block)
  uint32_t f1;      // Q6_K: offset of the unit's qh bytes in the block; Q1_0: of its bit word in the row
  uint32_t f2;      // Q6_K: offset of the unit's half of the scales in the block
  uint32_t sh;      // Q5_K: high-bit shift 2g; Q6_K: scale byte shift 8 lh
  uint32_t sel_a;   // K-quants: PRMT selector of the low scale/min bits
  uint32_t sel_h;   // K-quants: PRMT selector of the top two bits
  uint32_t mlo;     // K-quants: mask of the low bits (6 or 4 per value)
  uint32_t mhi;     // K-quants: mask of the moved top bits (0 for groups 0, 1)
};

template <int Q> FRC_DEVICE_INLINE UnitCtx make_ctx(int j, int b) {
  UnitCtx c{};
  c.j = j;
  c.blk = static_cast<uint32_t>(b * Fmt<Q>::TS);
  if constexpr (Q == kQ4_K) c.f0 = c.blk + 16u + 32u * j;
  if constexpr (Q == kQ5_K) c.f0 = c.blk + 48u + 32u * j;
  if constexpr (Q == kQ6_K) {
    const uint32_t half = static_cast<uint32_t>(j >> 1), lh = static_cast<uint32_t>(j & 1);
    c.f0 = 64u * half + 16u * lh;
    c.f1 = 128u + 32u * half + 16u * lh;
    c.f2 = 192u + 8u * half;
  }
  if constexpr (Q == kQ1_0) c.f1 = c.blk + 2u + 4u * j;
  if constexpr (Q == kQ4_K || Q == kQ5_K) {
    // Sub-blocks s0 = 2j, s1 = 2j + 1 use byte t0 = (2j) & 3 and t0 + 1 of
    // the scale words.  Groups 0, 1: sc = q[s] & 63 (word 0), m = q[s+4] & 63
    // (word 1).  Groups 2, 3: sc = (q[s+4] & 15) | (q[s-4] >> 6) << 4 (words
    // 2, 0), m = (q[s+4] >> 4) | (q[s] >> 6) << 4 (words 2, 1).  The PRMT
    // selectors pick byte t0 into bits 0-7 and byte t0+1 into bits 16-23
    // (selector value 7 reads a zero byte).
    const uint32_t t0 = static_cast<uint32_t>((2 * j) & 3);
    const uint32_t off = j >= 2 ? 4u : 0u;  // take the second PRMT source
    c.sel_a = (t0 + off) | (7u << 4) | ((t0 + 1u + off) << 8) | (7u << 12);
    c.sel_h = t0 | (7u << 4) | ((t0 + 1u) << 8) | (7u << 12);
    c.mlo = j >= 2 ? 0x000F000Fu : 0x003F003Fu;
    c.mhi = j >= 2 ? 0x00300030u : 0u;
    c.sh = static_cast<uint32_t>(2 * j);
  } else if constexpr (Q == kQ6_K) {
    c.sh = static_cast<uint32_t>(8 * (j & 1));
  }
  return c;
}

// The 6-bit scales and mins of sub-blocks 2g, 2g+1 of a K-quant block, as
// (sc0 | sc1 << 16) and (m0 | m1 << 16); s0..s2 hold scales[0..12].
FRC_DEVICE_INLINE void k_scales(const UnitCtx& c, uint32_t s0, uint32_t s1, uint32_t s2, uint32_t& sc,
                                uint32_t& mn) {
  const uint32_t a_sc = __byte_perm(s0, s2, c.sel_a);
  const uint32_t a_m = __byte_perm(s1, s2 >> 4, c.sel_a);
  const uint32_t h_sc = __byte_perm(s0, 0u, c.sel_h) >> 2;
  const uint32_t h_m = __byte_perm(s1, 0u, c.sel_h) >> 2;
  sc = (a_sc & c.mlo) | (h_sc & c.mhi);
  mn = (a_m & c.mlo) | (h_m & c.mhi);
}

template <int Q> struct UnitDotI8;

// Bounds: |xq| <= 32639.  Q4_K: |T| <= 32*15*32767 = 15.7e6 per sub-block,
// sc*T <= 991e6, two sub-blocks <= 1.98e9 < 2^31.
template <> struct UnitDotI8<kQ4_K> {
  // row: shared address of the row (16-byte aligned: 144-byte blocks)
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitX<kQ4_K>& x) {
    const uint4 hdr = lds128<0>(row + c.blk);
    const uint4 qa = lds128<0>(row + c.f0);
    const uint4 qb = lds128<16>(row + c.f0);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    // two accumulator chains per sum for instruction-level parallelism; the
    // high nibbles stay in place (16 * nibble, unsigned) and the factor 16 is
    // shifted out of the exact integer sum
    int lh0 = 0, ll0 = 0, hh0 = 0, hl0 = 0, lh1 = 0, ll1 = 0, hh1 = 0, hl1 = 0;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      lh0 = dp4a_ss(q[i] & 0x0F0F0F0Fu, x.xh[i], lh0);
      ll0 = dp4a_ss(q[i] & 0x0F0F0F0Fu, x.xl[i], ll0);
      hh0 = dp4a_us(q[i] & 0xF0F0F0F0u, x.xh[8 + i], hh0);
      hl0 = dp4a_us(q[i] & 0xF0F0F0F0u, x.xl[8 + i], hl0);
      lh1 = dp4a_ss(q[i + 1] & 0x0F0F0F0Fu, x.xh[i + 1], lh1);
      ll1 = dp4a_ss(q[i + 1] & 0x0F0F0F0Fu, x.xl[i + 1], ll1);
      hh1 = dp4a_us(q[i + 1] & 0xF0F0F0F0u, x.xh[9 + i], hh1);
      hl1 = dp4a_us(q[i + 1] & 0xF0F0F0F0u, x.xl[9 + i], hl1);
    }
    const int t0 = (lh0 + lh1) * 256 + (ll0 + ll1);
    const int t1 = ((hh0 + hh1) * 256 + (hl0 + hl1)) >> 4;  // exact: a multiple of 16
    uint32_t sc, mn;
    k_scales(c, hdr.y, hdr.z, hdr.w, sc, mn);
    const int u = static_cast<int>(sc & 0xFFFFu) * t0 + static_cast<int>(sc >> 16) * t1;
    const int v = static_cast<int>(mn & 0xFFFFu) * x.xsum[0] + static_cast<int>(mn >> 16) * x.xsum[1];
    const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
    return x.sx * (d * static_cast<float>(u) - dmin * static_cast<float>(v));
  }
};

// Q5_K: values nibble | bit << 4 in [0, 31]; |T| <= 32*31*32767 = 32.5e6,
// sc*T <= 2.05e9 is too close to 2^31 for two sub-blocks, so each sub-block
// is converted to fp32 separately.
template <> struct UnitDotI8<kQ5_K> {
  // row: shared address of the row (16-byte aligned: 176-byte blocks)
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitX<kQ5_K>& x) {
    const uint32_t blk = row + c.blk;
    const uint4 hdr = lds128<0>(blk);
    const uint4 ha = lds128<16>(blk);
    const uint4 hb = lds128<32>(blk);
    const uint4 qa = lds128<0>(row + c.f0);
    const uint4 qb = lds128<16>(row + c.f0);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const uint32_t h[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
    int lh = 0, ll = 0, hh = 0, hl = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = h[i] >> c.sh;  // bit 2g -> bit 0, bit 2g+1 -> bit 1
      const uint32_t lo = (q[i] & 0x0F0F0F0Fu) | ((b << 4) & 0x10101010u);
      const uint32_t hi = ((q[i] >> 4) & 0x0F0F0F0Fu) | ((b << 3) & 0x10101010u);
      lh = dp4a_ss(lo, x.xh[i], lh);
      ll = dp4a_ss(lo, x.xl[i], ll);
      hh = dp4a_ss(hi, x.xh[8 + i], hh);
      hl = dp4a_ss(hi, x.xl[8 + i], hl);
    }
    const int t0 = lh * 256 + ll;
    const int t1 = hh * 256 + hl;
    uint32_t sc, mn;
    k_scales(c, hdr.y, hdr.z, hdr.w, sc, mn);
    const float u = static_cast<float>(sc & 0xFFFFu) * static_cast<float>(t0) +
                    static_cast<float>(sc >> 16) * static_cast<float>(t1);
    const int v = static_cast<int>(mn & 0xFFFFu) * x.xsum[0] + static_cast<int>(mn >> 16) * x.xsum[1];
    const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
    return x.sx * (d * u - dmin * static_cast<float>(v));
  }
};

// Q6_K: u = nibble | 2 bits << 4 in [0, 63], weight (u - 32) * sc.
// Per quarter |T| <= 16*63*32767 = 33e6; T - 32 X fits int32; fp32 per quarter.
template <> struct UnitDotI8<kQ6_K> {
  // row: shared address of the row; 210-byte blocks are 2-byte aligned, so the
  // fields (at multiples of 4 inside the block) are read as aligned words
  // and funnel-shifted by the block's misalignment
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitX<kQ6_K>& x) {
    const uint32_t blk = row + c.blk;
    const uint32_t al = blk & ~3u, fs = (blk & 3u) * 8u;
    uint32_t qa[4], qb[4], qh[4], sw[2];
    lds_words_sh<4, 0>(al + c.f0, fs, qa);
    lds_words_sh<4, 32>(al + c.f0, fs, qb);
    lds_words_sh<4, 0>(al + c.f1, fs, qh);
    lds_words_sh<2, 0>(al + c.f2, fs, sw);
    int sh[4] = {0, 0, 0, 0}, sl[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u0 = (qa[i] & 0x0F0F0F0Fu) | ((qh[i] << 4) & 0x30303030u);
      const uint32_t u1 = (qb[i] & 0x0F0F0F0Fu) | ((qh[i] << 2) & 0x30303030u);
      const uint32_t u2 = ((qa[i] >> 4) & 0x0F0F0F0Fu) | (qh[i] & 0x30303030u);
      const uint32_t u3 = ((qb[i] >> 4) & 0x0F0F0F0Fu) | ((qh[i] >> 2) & 0x30303030u);
      sh[0] = dp4a_ss(u0, x.xh[i], sh[0]);
      sl[0] = dp4a_ss(u0, x.xl[i], sl[0]);
      sh[1] = dp4a_ss(u1, x.xh[4 + i], sh[1]);
      sl[1] = dp4a_ss(u1, x.xl[4 + i], sl[1]);
      sh[2] = dp4a_ss(u2, x.xh[8 + i], sh[2]);
      sl[2] = dp4a_ss(u2, x.xl[8 + i], sl[2]);
      sh[3] = dp4a_ss(u3, x.xh[12 + i], sh[3]);
      sl[3] = dp4a_ss(u3, x.xl[12 + i], sl[3]);
    }
    // scales[8 half + 2 r + lh], r = quarter: bytes lh, lh+2 of sw[0], sw[1]
    const uint32_t sa = sw[0] >> c.sh, sb = sw[1] >> c.sh;
    const float s0 = static_cast<float>(static_cast<int>(sa << 24) >> 24);
    const float s1 = static_cast<float>(static_cast<int>(sa << 8) >> 24);
    const float s2 = static_cast<float>(static_cast<int>(sb << 24) >> 24);
    const float s3 = static_cast<float>(static_cast<int>(sb << 8) >> 24);
    const float w0 = static_cast<float>(sh[0] * 256 + sl[0] - 32 * x.xsum[0]);
    const float w1 = static_cast<float>(sh[1] * 256 + sl[1] - 32 * x.xsum[1]);
    const float w2 = static_cast<float>(sh[2] * 256 + sl[2] - 32 * x.xsum[2]);
    const float w3 = static_cast<float>(sh[3] * 256 + sl[3] - 32 * x.xsum[3]);
    const float d = half_bits_to_float(lds16<208>(blk));
    return x.sx * d * ((s0 * w0 + s1 * w1) + (s2 * w2 + s3 * w3));
  }
};

// Q8_0: signed quants; |T| <= 32*127*32767 = 133e6.
template <> struct UnitDotI8<kQ8_0> {
  // row: shared address of the row; 34-byte blocks are 2-byte aligned
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitX<kQ8_0>& x) {
    const uint32_t blk = row + c.blk, qs = blk + 2u;
    uint32_t q[8];
    lds_words_sh<8, 0>(qs & ~3u, (qs & 3u) * 8u, q);
    int sh = 0, sl = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sh = dp4a_ss(q[i], x.xh[i], sh);
      sl = dp4a_ss(q[i], x.xl[i], sl);
    }
    const float d = half_bits_to_float(lds16<0>(blk));
    return x.sx * d * static_cast<float>(sh * 256 + sl);
  }
};

// Q1_0: sum(s_i x_i) = 2 * sum(x_i, bit set) - sum(x_i).  Bits are spread to
// bytes four at a time: (nibble * 0x00204081) & 0x01010101 puts bit b of the
// nibble in byte b.
template <> struct UnitDotI8<kQ1_0> {
  // row: shared address of the row; 18-byte blocks are 2-byte aligned
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitX<kQ1_0>& x) {
    const uint32_t bw = row + c.f1;
    uint32_t bits1[1];
    lds_words_sh<1, 0>(bw & ~3u, (bw & 3u) * 8u, bits1);
    const uint32_t bits = bits1[0];
    int sh = 0, sl = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = (((bits >> (4 * i)) & 0xFu) * 0x00204081u) & 0x01010101u;
      sh = dp4a_ss(b, x.xh[i], sh);
      sl = dp4a_ss(b, x.xl[i], sl);
    }
    const float d = half_bits_to_float(lds16<0>(row + c.blk));
    return x.sx * d * static_cast<float>(2 * (sh * 256 + sl) - x.xsum[0]);
  }
};

}  // namespace frc
