// GGUF block formats on the device: geometry, bit-exact dequantisation and the
// exact decode of one "unit" used by the batched fp32 GEMV.
//
// Block layouts and element order follow the reference decoders in
// src/flatrun/dequant/gguf.py (Q8_0 :112-127, Q4_K :166-220, Q5_K :223-263,
// Q1_0 :266-299, Q6_K :365-420; scale/min unpack :135-163).
//
// A "unit" here is the slice of one block that one thread of the batched
// fp32 kernel (gemv_xb) decodes into registers: NRUN runs of 16 consecutive
// elements of the row, so its activations load as float4s.  The batch-1
// kernel's units (64 or 32 elements) are defined in units_dp4a.cuh.
#pragma once

#include "frc_common.cuh"

namespace frc {

enum Quant : int { kQ8_0 = 8, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14, kQ1_0 = 41 };

template <int Q> struct Fmt;

template <> struct Fmt<kQ8_0> { static constexpr int QK = 32,  TS = 34,  UPB = 1, NRUN = 2; };
template <> struct Fmt<kQ4_K> { static constexpr int QK = 256, TS = 144, UPB = 8, NRUN = 2; };
template <> struct Fmt<kQ5_K> { static constexpr int QK = 256, TS = 176, UPB = 8, NRUN = 2; };
template <> struct Fmt<kQ6_K> { static constexpr int QK = 256, TS = 210, UPB = 4, NRUN = 4; };
template <> struct Fmt<kQ1_0> { static constexpr int QK = 128, TS = 18,  UPB = 4, NRUN = 2; };

// ---------------------------------------------------------------------------
// 6-bit scale/min unpack of the K-quants (gguf.py:135-163).
// ---------------------------------------------------------------------------
FRC_DEVICE_INLINE void scale_min_k4(int j, const uint8_t* q, uint32_t& sc, uint32_t& m) {
  if (j < 4) {
    sc = q[j] & 63u;
    m = q[j + 4] & 63u;
  } else {
    sc = (q[j + 4] & 0x0Fu) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// Same, from the three little-endian words holding scales[0..12].
FRC_DEVICE_INLINE void scale_min_k4_words(int j, uint32_t s0, uint32_t s1, uint32_t s2, float& sc,
                                          float& m) {
  const uint32_t t = static_cast<uint32_t>(j & 3) * 8u;
  const uint32_t b0 = (s0 >> t) & 0xFFu, b1 = (s1 >> t) & 0xFFu, b2 = (s2 >> t) & 0xFFu;
  uint32_t vs, vm;
  if (j < 4) {
    vs = b0 & 63u;
    vm = b1 & 63u;
  } else {
    vs = (b2 & 0x0Fu) | ((b0 >> 6) << 4);
    vm = (b2 >> 4) | ((b1 >> 6) << 4);
  }
  sc = static_cast<float>(vs);
  m = static_cast<float>(vm);
}

// ---------------------------------------------------------------------------
// Bit-exact dequantisation of element e of a block.  The arithmetic is the
// reference NumPy expression, operation by operation, with no contraction.
// ---------------------------------------------------------------------------
template <int Q> FRC_DEVICE_INLINE float dequant_elem(const uint8_t* blk, int e);

template <> FRC_DEVICE_INLINE float dequant_elem<kQ8_0>(const uint8_t* blk, int e) {
  // qs * d (gguf.py:126-127)
  const float d = half_bits_to_float(ld_u16(blk));
  const float q = static_cast<float>(static_cast<int8_t>(blk[2 + e]));
  return __fmul_rn(q, d);
}

template <> FRC_DEVICE_INLINE float dequant_elem<kQ4_K>(const uint8_t* blk, int e) {
  // ((d * sc) * q) - (dmin * m) in fp32 (gguf.py:210-219)
  const int g = e >> 6, r = e & 63, hi = r >> 5, i = r & 31;
  const float d = half_bits_to_float(ld_u16(blk));
  const float dmin = half_bits_to_float(ld_u16(blk + 2));
  uint32_t sc, m;
  scale_min_k4(2 * g + hi, blk + 4, sc, m);
  const uint32_t byte = blk[16 + g * 32 + i];
  const float q = static_cast<float>(hi ? (byte >> 4) : (byte & 0x0Fu));
  return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), q),
                   __fmul_rn(dmin, static_cast<float>(m)));
}

template <> FRC_DEVICE_INLINE float dequant_elem<kQ5_K>(const uint8_t* blk, int e) {
  // The reference adds np.where(..., 16.0, 0.0) (float64) to the fp32 nibble,
  // so (d*sc) [fp32] * v - (dmin*m) [fp32] is evaluated in float64 and then
  // stored to fp32 (gguf.py:257-262).
  const int g = e >> 6, r = e & 63, hi = r >> 5, i = r & 31;
  const float d = half_bits_to_float(ld_u16(blk));
  const float dmin = half_bits_to_float(ld_u16(blk + 2));
  uint32_t sc, m;
  scale_min_k4(2 * g + hi, blk + 4, sc, m);
  const uint32_t byte = blk[48 + g * 32 + i];
  const uint32_t qh = blk[16 + i];
  uint32_t v = hi ? (byte >> 4) : (byte & 0x0Fu);
  if ((qh >> (2 * g + hi)) & 1u) v += 16u;
  const double ds = static_cast<double>(__fmul_rn(d, static_cast<float>(sc)));
  const double dm = static_cast<double>(__fmul_rn(dmin, static_cast<float>(m)));
  return __double2float_rn(__dsub_rn(__dmul_rn(ds, static_cast<double>(v)), dm));
}

template <> FRC_DEVICE_INLINE float dequant_elem<kQ6_K>(const uint8_t* blk, int e) {
  // (d * sc) * q with q = nibble | (2 bits << 4) - 32 (gguf.py:400-419)
  const int half = e >> 7, r = e & 127, qq = r >> 5, l = r & 31;
  const uint32_t qlb = blk[half * 64 + ((qq & 1) ? 32 : 0) + l];
  const uint32_t nib = (qq & 2) ? (qlb >> 4) : (qlb & 0x0Fu);
  const uint32_t h2 = (blk[128 + half * 32 + l] >> (2 * qq)) & 3u;
  const float q = __fsub_rn(__fadd_rn(static_cast<float>(nib), static_cast<float>(h2 << 4)), 32.0f);
  const float sc = static_cast<float>(static_cast<int8_t>(blk[192 + half * 8 + 2 * qq + (l >> 4)]));
  const float d = half_bits_to_float(ld_u16(blk + 208));
  return __fmul_rn(__fmul_rn(d, sc), q);
}

template <> FRC_DEVICE_INLINE float dequant_elem<kQ1_0>(const uint8_t* blk, int e) {
  // (+1 | -1) * d, bit e%8 of byte e/8, LSB first (gguf.py:291-298)
  const float d = half_bits_to_float(ld_u16(blk));
  const float s = ((blk[2 + (e >> 3)] >> (e & 7)) & 1u) ? 1.0f : -1.0f;
  return __fmul_rn(s, d);
}

// ---------------------------------------------------------------------------
// Units: element positions.  run_start(j, r) is the offset, inside the block,
// of the r-th 16-element run of unit j.
// ---------------------------------------------------------------------------
template <int Q> FRC_DEVICE_INLINE int run_start(int j, int r);
// Q8_0: one unit = the block's 32 elements.
template <> FRC_DEVICE_INLINE int run_start<kQ8_0>(int, int r) { return 16 * r; }
// Q4_K/Q5_K unit j = (group g = j/2, half h = j%2): 16 bytes of qs whose low
// nibbles are elements 64g+16h+[0,16) and high nibbles 64g+32+16h+[0,16).
template <> FRC_DEVICE_INLINE int run_start<kQ4_K>(int j, int r) { return 64 * (j >> 1) + 32 * r + 16 * (j & 1); }
template <> FRC_DEVICE_INLINE int run_start<kQ5_K>(int j, int r) { return 64 * (j >> 1) + 32 * r + 16 * (j & 1); }
// Q6_K unit j = (half = j/2, l-range lh = j%2): ql[l], ql[l+32], qh[l] for
// l in 16lh+[0,16) give elements 128half + 32r + 16lh + [0,16), r = quarter.
template <> FRC_DEVICE_INLINE int run_start<kQ6_K>(int j, int r) { return 128 * (j >> 1) + 32 * r + 16 * (j & 1); }
// Q1_0 unit j: sign bytes 4j..4j+3, elements 32j + [0,32).
template <> FRC_DEVICE_INLINE int run_start<kQ1_0>(int j, int r) { return 32 * j + 16 * r; }

// ---------------------------------------------------------------------------
// Exact decode of a unit's elements (used by the batched kernel, which shares
// one decode across up to 16 activation columns).  out[r*16 + i] is element
// run_start(j, r) + i.  Products are rounded per element as in dequant_elem
// except Q5_K, where the fp32 expression is used (within 1 ulp of the
// float64 reference; the batched GEMV is checked by tolerance, not bits).
// ---------------------------------------------------------------------------
template <int Q> struct UnitDecode;

template <> struct UnitDecode<kQ4_K> {
  static FRC_DEVICE_INLINE void run(const uint8_t* blk, int j, float* out) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const uint4 qs = *reinterpret_cast<const uint4*>(blk + 16 + 32 * (j >> 1) + 16 * (j & 1));
    const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
    float sc0, m0, sc1, m1;
    scale_min_k4_words(2 * (j >> 1), hdr.y, hdr.z, hdr.w, sc0, m0);
    scale_min_k4_words(2 * (j >> 1) + 1, hdr.y, hdr.z, hdr.w, sc1, m1);
    const float a0 = d * sc0, b0 = dmin * m0, a1 = d * sc1, b1 = dmin * m1;
    const uint32_t q[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t byte = (q[i >> 2] >> (8 * (i & 3))) & 0xFFu;
      out[i] = a0 * static_cast<float>(byte & 0x0Fu) - b0;
      out[16 + i] = a1 * static_cast<float>(byte >> 4) - b1;
    }
  }
};

template <> struct UnitDecode<kQ5_K> {
  static FRC_DEVICE_INLINE void run(const uint8_t* blk, int j, float* out) {
    const int g = j >> 1, h = j & 1;
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const uint4 qh = *reinterpret_cast<const uint4*>(blk + 16 + 16 * h);
    const uint4 qs = *reinterpret_cast<const uint4*>(blk + 48 + 32 * g + 16 * h);
    const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
    float sc0, m0, sc1, m1;
    scale_min_k4_words(2 * g, hdr.y, hdr.z, hdr.w, sc0, m0);
    scale_min_k4_words(2 * g + 1, hdr.y, hdr.z, hdr.w, sc1, m1);
    const float a0 = d * sc0, b0 = dmin * m0, a1 = d * sc1, b1 = dmin * m1;
    const uint32_t q[4] = {qs.x, qs.y, qs.z, qs.w};
    const uint32_t hb[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t byte = (q[i >> 2] >> (8 * (i & 3))) & 0xFFu;
      const uint32_t hbyte = (hb[i >> 2] >> (8 * (i & 3))) & 0xFFu;
      const uint32_t v0 = (byte & 0x0Fu) | (((hbyte >> (2 * g)) & 1u) << 4);
      const uint32_t v1 = (byte >> 4) | (((hbyte >> (2 * g + 1)) & 1u) << 4);
      out[i] = a0 * static_cast<float>(v0) - b0;
      out[16 + i] = a1 * static_cast<float>(v1) - b1;
    }
  }
};

template <> struct UnitDecode<kQ6_K> {
  static FRC_DEVICE_INLINE void run(const uint8_t* blk, int j, float* out) {
    const int half = j >> 1, lh = j & 1;
    uint32_t qa[4], qb[4], qh[4], sw[2];
    lds_words_a2<4>(blk + 64 * half + 16 * lh, qa);
    lds_words_a2<4>(blk + 64 * half + 32 + 16 * lh, qb);
    lds_words_a2<4>(blk + 128 + 32 * half + 16 * lh, qh);
    lds_words_a2<2>(blk + 192 + 8 * half, sw);
    const float d = half_bits_to_float(ld_u16(blk + 208));
    const uint32_t sA = sw[0] >> (8 * lh), sB = sw[1] >> (8 * lh);
    const float s[4] = {d * static_cast<float>(static_cast<int8_t>(sA & 0xFF)),
                        d * static_cast<float>(static_cast<int8_t>((sA >> 16) & 0xFF)),
                        d * static_cast<float>(static_cast<int8_t>(sB & 0xFF)),
                        d * static_cast<float>(static_cast<int8_t>((sB >> 16) & 0xFF))};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int sh = 8 * (i & 3);
      const uint32_t a = (qa[i >> 2] >> sh) & 0xFFu, b = (qb[i >> 2] >> sh) & 0xFFu;
      const uint32_t hh = (qh[i >> 2] >> sh) & 0xFFu;
      out[i] = s[0] * (static_cast<float>((a & 0x0Fu) | ((hh & 3u) << 4)) - 32.0f);
      out[16 + i] = s[1] * (static_cast<float>((b & 0x0Fu) | (((hh >> 2) & 3u) << 4)) - 32.0f);
      out[32 + i] = s[2] * (static_cast<float>((a >> 4) | (((hh >> 4) & 3u) << 4)) - 32.0f);
      out[48 + i] = s[3] * (static_cast<float>((b >> 4) | (((hh >> 6) & 3u) << 4)) - 32.0f);
    }
  }
};

template <> struct UnitDecode<kQ8_0> {
  static FRC_DEVICE_INLINE void run(const uint8_t* blk, int, float* out) {
    uint32_t q[8];
    lds_words_a2<8>(blk + 2, q);
    const float d = half_bits_to_float(ld_u16(blk));
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      out[i] = d * static_cast<float>(static_cast<int8_t>((q[i >> 2] >> (8 * (i & 3))) & 0xFFu));
    }
  }
};

template <> struct UnitDecode<kQ1_0> {
  static FRC_DEVICE_INLINE void run(const uint8_t* blk, int j, float* out) {
    const uint32_t bits = ld_u32_a2(blk + 2 + 4 * j);
    const float d = half_bits_to_float(ld_u16(blk));
#pragma unroll
    for (int i = 0; i < 32; ++i) out[i] = ((bits >> i) & 1u) ? d : -d;
  }
};

}  // namespace frc
