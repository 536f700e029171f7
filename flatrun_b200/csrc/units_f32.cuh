// fp32-activation units for the batch-1 GEMV: the reference's arithmetic.
//
// The reference multiplies dequantised fp32 weights by fp32 activations and
// sums in fp32 (src/flatrun_native/kernels/q4_k.h:153-184, q8_0.h:36-50; the
// NumPy path is dequant + fp32 BLAS, runtime/backend.py:180-213).  These
// units do the same: every activation stays an fp32 value, every product is
// an fp32 multiply-add against that value, and every sum is fp32.  Only the
// order of the algebra differs: a block's scale (and its min, offset or sign
// identity) is applied once per scale group to the group's sum of q * x
// instead of to every weight, which is exact in real arithmetic.
//
// A unit is the slice of one block a thread owns (the geometry of the integer
// units, I8<Q>: 64 elements for the K-quants, 32 for Q8_0 and Q1_0), with its
// activations in registers for the whole launch.  Quant values become fp32
// without an integer conversion instruction, by a byte permute into the bits
// of a float:
//   * "unit" encoding: a value u < 128 placed, ORed with 0x80, in bits 16-23
//     of 1.0f reads as 1 + u/128 exactly; with A = sum((1 + u/128) x) and
//     X = sum(x) over a group, sum(u x) = 128 (A - X);
//   * "magic" encoding: a byte u in bits 0-7 of 2^23 reads as 2^23 + u
//     exactly; one packed subtraction leaves u, and products are exact.
// The second costs an extra FADD2 per two elements, the first none; each
// format uses the cheaper one its value range allows (unit needs u < 128).
#pragma once

#include "units_dp4a.cuh"

namespace frc {

// Activations of one unit: E fp32 values in unit order (element i of unit j
// is element i8_pos<Q>(j, i) of block b) and their sum over every scale group
// (E / NG consecutive values).
template <int Q>
struct UnitXF {
  static constexpr int E = I8<Q>::E, NG = I8<Q>::NG, GE = E / NG;
  float x[E];
  float xs[NG];
  const float* mul_ = nullptr;  // silu(x) * mul activations (see load)
  int j_ = 0;
  int64_t b_ = 0;

  // Unit j of block b.  Every 16 consecutive unit elements are 16 consecutive
  // elements of x, so the unit loads as E/4 float4s, all issued before any
  // is used; finish() applies the SwiGLU and sums() forms the group sums.  With `mul` the
  // activations are silu(x) * mul, formed in finish() as the reference does
  // (s = 1 / (1 + exp(-gate)); s * gate * up, qwen2.py:1690-1751).
  FRC_DEVICE_INLINE void load(const float* xg, const float* mul, int64_t b, int j) {
    const float* blk = xg + b * Fmt<Q>::QK;
#pragma unroll
    for (int r = 0; r < E / 16; ++r) {
      const float4* src = reinterpret_cast<const float4*>(blk + i8_pos<Q>(j, 16 * r));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = __ldg(src + q);
        x[16 * r + 4 * q] = v.x;
        x[16 * r + 4 * q + 1] = v.y;
        x[16 * r + 4 * q + 2] = v.z;
        x[16 * r + 4 * q + 3] = v.w;
      }
    }
    mul_ = mul ? mul + b * Fmt<Q>::QK : nullptr;
    j_ = j;
    b_ = b;
  }
  // The unit's elements of a vector laid out like x (weights of an RMSNorm).
  FRC_DEVICE_INLINE float4 like_x(const float* v, int r, int q) const {
    return __ldg(reinterpret_cast<const float4*>(v + b_ * Fmt<Q>::QK + i8_pos<Q>(j_, 16 * r)) + q);
  }
  FRC_DEVICE_INLINE float sum_squares() const {
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      s0 = fmaf(x[e], x[e], s0);
      s1 = fmaf(x[e + 1], x[e + 1], s1);
    }
    return s0 + s1;
  }
  // x <- (x * inv) * w: the RMSNorm of the reference (qwen2.py:365-378).
  FRC_DEVICE_INLINE void normalise(float inv, const float* w) {
#pragma unroll
    for (int r = 0; r < E / 16; ++r) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 g = like_x(w, r, q);
        const float gs[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) x[16 * r + 4 * q + e] = (x[16 * r + 4 * q + e] * inv) * gs[e];
      }
    }
  }
  // silu(x) * mul when the unit was loaded with `mul`.
  FRC_DEVICE_INLINE void finish() {
    if (mul_) {
#pragma unroll
      for (int r = 0; r < E / 16; ++r) {
        const float4* src = reinterpret_cast<const float4*>(mul_ + i8_pos<Q>(j_, 16 * r));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 u = __ldg(src + q);
          const float us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float g = x[16 * r + 4 * q + e];
            const float s = 1.0f / (1.0f + expf(-g));
            x[16 * r + 4 * q + e] = (s * g) * us[e];
          }
        }
      }
    }
  }
  // The group sums (after any transform of x).
  FRC_DEVICE_INLINE void sums() {
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int e = 0; e < GE; e += 2) {
        s0 += x[g * GE + e];
        s1 += x[g * GE + e + 1];
      }
      xs[g] = s0 + s1;
    }
  }
  FRC_DEVICE_INLINE void zero() {
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g) xs[g] = 0.f;
    mul_ = nullptr;
  }
};

// sum over the 4 bytes of w (each 0x80 | u, u < 128) of (1 + u/128) * x[0..3],
// into two accumulator lanes.
FRC_DEVICE_INLINE float2 fma4_unit(uint32_t w, const float* x, float2 acc) {
  acc = __ffma2_rn(make_float2(byte_as_unit_float<0>(w), byte_as_unit_float<1>(w)), make_float2(x[0], x[1]), acc);
  acc = __ffma2_rn(make_float2(byte_as_unit_float<2>(w), byte_as_unit_float<3>(w)), make_float2(x[2], x[3]), acc);
  return acc;
}

// sum over the 4 bytes u of w of (u + bias) * x[0..3], the bytes turned into
// exact floats through 2^23 + u; `bias2` holds -(2^23 - bias) twice.
FRC_DEVICE_INLINE float2 fma4_magic(uint32_t w, const float* x, float2 bias2, float2 acc) {
  const float2 f01 = __fadd2_rn(make_float2(byte_as_magic_float<0>(w), byte_as_magic_float<1>(w)), bias2);
  const float2 f23 = __fadd2_rn(make_float2(byte_as_magic_float<2>(w), byte_as_magic_float<3>(w)), bias2);
  acc = __ffma2_rn(f01, make_float2(x[0], x[1]), acc);
  acc = __ffma2_rn(f23, make_float2(x[2], x[3]), acc);
  return acc;
}

FRC_DEVICE_INLINE float lanes(float2 a, float2 b) { return (a.x + b.x) + (a.y + b.y); }

template <int Q> struct UnitDotF32;

// Q4_K unit j = group g: qs bytes [32g, 32g + 32) of the block; low nibbles are
// elements 64g + [0, 32) (sub-block 2g), high nibbles 64g + 32 + [0, 32)
// (sub-block 2g+1).  Low nibbles use the unit encoding; high nibbles stay in
// place (16 * h < 256, magic encoding) and the factor 16 moves into the scale.
template <> struct UnitDotF32<kQ4_K> {
  // row: shared address of the row (16-byte aligned: 144-byte blocks)
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitXF<kQ4_K>& x) {
    const uint4 hdr = lds128<0>(row + c.blk);
    const uint4 qa = lds128<0>(row + c.f0);
    const uint4 qb = lds128<16>(row + c.f0);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const float2 m23 = make_float2(-8388608.0f, -8388608.0f);
    float2 l0 = make_float2(0.f, 0.f), l1 = l0, h0 = l0, h1 = l0;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      l0 = fma4_unit((q[i] & 0x0F0F0F0Fu) | 0x80808080u, x.x + 4 * i, l0);
      h0 = fma4_magic(q[i] & 0xF0F0F0F0u, x.x + 32 + 4 * i, m23, h0);
      l1 = fma4_unit((q[i + 1] & 0x0F0F0F0Fu) | 0x80808080u, x.x + 4 * i + 4, l1);
      h1 = fma4_magic(q[i + 1] & 0xF0F0F0F0u, x.x + 36 + 4 * i, m23, h1);
    }
    const float s_lo = 128.0f * (lanes(l0, l1) - x.xs[0]);  // sum(lo * x)
    const float s_hi16 = lanes(h0, h1);                      // sum(16 hi * x)
    uint32_t sc, mn;
    k_scales(c, hdr.y, hdr.z, hdr.w, sc, mn);
    const float sc0 = static_cast<float>(sc & 0xFFFFu), sc1 = static_cast<float>(sc >> 16) * 0.0625f;
    const float m0 = static_cast<float>(mn & 0xFFFFu), m1 = static_cast<float>(mn >> 16);
    const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
    return d * (sc0 * s_lo + sc1 * s_hi16) - dmin * (m0 * x.xs[0] + m1 * x.xs[1]);
  }
};

// Q5_K: values nibble | bit << 4 in [0, 31] (the 5th bit of element l of
// sub-block s is bit s of qh byte l), unit encoding for both sub-blocks.
template <> struct UnitDotF32<kQ5_K> {
  // row: shared address of the row (16-byte aligned: 176-byte blocks)
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitXF<kQ5_K>& x) {
    const uint32_t blk = row + c.blk;
    const uint4 hdr = lds128<0>(blk);
    const uint4 ha = lds128<16>(blk);
    const uint4 hb = lds128<32>(blk);
    const uint4 qa = lds128<0>(row + c.f0);
    const uint4 qb = lds128<16>(row + c.f0);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const uint32_t h[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
    float2 l0 = make_float2(0.f, 0.f), l1 = l0, h0 = l0, h1 = l0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = h[i] >> c.sh;  // bit 2g -> bit 0, bit 2g+1 -> bit 1 of every byte
      const uint32_t lo = (q[i] & 0x0F0F0F0Fu) | ((b << 4) & 0x10101010u) | 0x80808080u;
      const uint32_t hi = ((q[i] >> 4) & 0x0F0F0F0Fu) | ((b << 3) & 0x10101010u) | 0x80808080u;
      if (i & 1) {
        l1 = fma4_unit(lo, x.x + 4 * i, l1);
        h1 = fma4_unit(hi, x.x + 32 + 4 * i, h1);
      } else {
        l0 = fma4_unit(lo, x.x + 4 * i, l0);
        h0 = fma4_unit(hi, x.x + 32 + 4 * i, h0);
      }
    }
    const float s_lo = 128.0f * (lanes(l0, l1) - x.xs[0]);
    const float s_hi = 128.0f * (lanes(h0, h1) - x.xs[1]);
    uint32_t sc, mn;
    k_scales(c, hdr.y, hdr.z, hdr.w, sc, mn);
    const float sc0 = static_cast<float>(sc & 0xFFFFu), sc1 = static_cast<float>(sc >> 16);
    const float m0 = static_cast<float>(mn & 0xFFFFu), m1 = static_cast<float>(mn >> 16);
    const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
    return d * (sc0 * s_lo + sc1 * s_hi) - dmin * (m0 * x.xs[0] + m1 * x.xs[1]);
  }
};

// Q6_K unit j = (half, lh): quarter r holds elements 128 half + 32 r + 16 lh
// + [0, 16); u = nibble | 2 bits << 4 in [0, 63] (unit encoding), weight
// (u - 32) * sc * d with one int8 scale per quarter.
template <> struct UnitDotF32<kQ6_K> {
  // row: shared address of the row; 210-byte blocks are 2-byte aligned, so
  // the fields are read as aligned words and funnel-shifted
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitXF<kQ6_K>& x) {
    const uint32_t blk = row + c.blk;
    const uint32_t al = blk & ~3u, fs = (blk & 3u) * 8u;
    uint32_t qa[4], qb[4], qh[4], sw[2];
    lds_words_sh<4, 0>(al + c.f0, fs, qa);
    lds_words_sh<4, 32>(al + c.f0, fs, qb);
    lds_words_sh<4, 0>(al + c.f1, fs, qh);
    lds_words_sh<2, 0>(al + c.f2, fs, sw);
    float2 a[4][2];
#pragma unroll
    for (int r = 0; r < 4; ++r) a[r][0] = a[r][1] = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t u0 = (qa[i] & 0x0F0F0F0Fu) | ((qh[i] << 4) & 0x30303030u) | 0x80808080u;
      const uint32_t u1 = (qb[i] & 0x0F0F0F0Fu) | ((qh[i] << 2) & 0x30303030u) | 0x80808080u;
      const uint32_t u2 = ((qa[i] >> 4) & 0x0F0F0F0Fu) | (qh[i] & 0x30303030u) | 0x80808080u;
      const uint32_t u3 = ((qb[i] >> 4) & 0x0F0F0F0Fu) | ((qh[i] >> 2) & 0x30303030u) | 0x80808080u;
      a[0][i & 1] = fma4_unit(u0, x.x + 4 * i, a[0][i & 1]);
      a[1][i & 1] = fma4_unit(u1, x.x + 16 + 4 * i, a[1][i & 1]);
      a[2][i & 1] = fma4_unit(u2, x.x + 32 + 4 * i, a[2][i & 1]);
      a[3][i & 1] = fma4_unit(u3, x.x + 48 + 4 * i, a[3][i & 1]);
    }
    // sum((u - 32) x) = 128 (A - X) - 32 X per quarter; scales[8 half + 2 r + lh]
    // are bytes lh, lh + 2 of sw[0] (quarters 0, 1) and sw[1] (2, 3)
    const uint32_t sa = sw[0] >> c.sh, sb = sw[1] >> c.sh;
    const float s0 = static_cast<float>(static_cast<int>(sa << 24) >> 24);
    const float s1 = static_cast<float>(static_cast<int>(sa << 8) >> 24);
    const float s2 = static_cast<float>(static_cast<int>(sb << 24) >> 24);
    const float s3 = static_cast<float>(static_cast<int>(sb << 8) >> 24);
    float t[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) t[r] = 128.0f * (lanes(a[r][0], a[r][1]) - x.xs[r]) - 32.0f * x.xs[r];
    const float d = half_bits_to_float(lds16<208>(blk));
    return d * ((s0 * t[0] + s1 * t[1]) + (s2 * t[2] + s3 * t[3]));
  }
};

// Q8_0: signed quants, magic encoding of q + 128 and an exact subtraction of
// 2^23 + 128.
template <> struct UnitDotF32<kQ8_0> {
  // row: shared address of the row; 34-byte blocks are 2-byte aligned
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitXF<kQ8_0>& x) {
    const uint32_t blk = row + c.blk, qs = blk + 2u;
    uint32_t q[8];
    lds_words_sh<8, 0>(qs & ~3u, (qs & 3u) * 8u, q);
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    float2 a0 = make_float2(0.f, 0.f), a1 = a0;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      a0 = fma4_magic(q[i] ^ 0x80808080u, x.x + 4 * i, bias, a0);
      a1 = fma4_magic(q[i + 1] ^ 0x80808080u, x.x + 4 * i + 4, bias, a1);
    }
    const float d = half_bits_to_float(lds16<0>(blk));
    return d * lanes(a0, a1);
  }
};

// Q1_0: sum(s_i x_i) with s = +-1 is 2 * sum(x_i, bit set) - sum(x_i).  Four
// bits at a time are spread to bytes ((nibble * 0x00204081) & 0x01010101 puts
// bit b in byte b) and enter through the magic encoding.
template <> struct UnitDotF32<kQ1_0> {
  // row: shared address of the row; 18-byte blocks are 2-byte aligned
  static FRC_DEVICE_INLINE float dot(uint32_t row, const UnitCtx& c, const UnitXF<kQ1_0>& x) {
    const uint32_t bw = row + c.f1;
    uint32_t bits1[1];
    lds_words_sh<1, 0>(bw & ~3u, (bw & 3u) * 8u, bits1);
    const uint32_t bits = bits1[0];
    const float2 m23 = make_float2(-8388608.0f, -8388608.0f);
    float2 a0 = make_float2(0.f, 0.f), a1 = a0;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const uint32_t b0 = (((bits >> (4 * i)) & 0xFu) * 0x00204081u) & 0x01010101u;
      const uint32_t b1 = (((bits >> (4 * i + 4)) & 0xFu) * 0x00204081u) & 0x01010101u;
      a0 = fma4_magic(b0, x.x + 4 * i, m23, a0);
      a1 = fma4_magic(b1, x.x + 4 * i + 4, m23, a1);
    }
    const float d = half_bits_to_float(lds16<0>(row + c.blk));
    return d * (2.0f * lanes(a0, a1) - x.xs[0]);
  }
};

}  // namespace frc
