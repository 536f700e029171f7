// Batch-1 GEMV on the tensor cores with exact fp32 activations: gemv_tc1<Q>
// (Q4_K, and Q5_K with its fifth bits joined to the nibbles, see tc1_sb).
//
// The reference multiplies dequantised fp32 weights by fp32 x and sums in
// fp32 (src/flatrun_native/kernels/q4_k.h:153-184; the NumPy path is dequant
// + fp32 BLAS).  This kernel computes the same sums with every product exact:
//   * a Q4_K weight is d * sc * q - dmin * m (q a nibble, sc and m 6-bit
//     integers of its 32-element sub-block, d and dmin fp16 per 256-element
//     super-block).  q * sc <= 945 is an integer, exact in fp16;
//   * x is scaled by a power of two per super-block (s, so that |x s| < 2^15)
//     and written as the sum of three fp16 terms, hi + mid + lo, each the
//     round-to-nearest fp16 of what the previous terms leave: 33 significand
//     bits cover fp32's 24, so the three terms sum to x s exactly (short of
//     fp16 underflow for elements below 2^-9 of the super-block's largest,
//     whose lost bits are below 2^-39 of that largest element);
//   * one mma.sync m16n8k16 (f16 x f16, fp32 accumulate) multiplies 16 rows
//     of q * sc by the three terms in columns 0..2 of B; fp16 x fp16 products
//     (11 x 11 significant bits) are exact in fp32, so the MMA's column sums
//     are fp32 sums of exact products, as the reference's dot is;
//   * per super-block and row, y += d / s * (hi + mid + lo column sums) -
//     dmin * sum_j m_j xs_j, with xs_j the fp32 sum of x over sub-block j:
//     the reference's algebra with the scales applied per group instead of
//     per weight.
//
// Why warp-level mma.sync and not tcgen05 here: at batch 1 the products are
// a few percent of the tensor pipe, and what costs is turning raw quant
// bytes into MMA operands.  mma.sync takes A from registers, so each thread
// converts its bytes (a mask and one fp16 FMA per two weights, no shared-
// memory round trip for the dequantised tile) straight into its fragment;
// tcgen05 would need the converted tile written to shared memory or TMEM
// and a single-thread issue per tile.
//
// Operand layout (m16n8k16, thread (g = lane / 4, t = lane % 4)):
//   * A: rows g and g + 8 of a 16-row MMA tile; thread t converts quant bytes
//     [32t, 32t + 32) of each super-block's qs (its chunk t: low nibbles are
//     sub-block 2t, high nibbles sub-block 2t + 1).  Word i of the chunk gives
//     two MMAs: low nibbles (bytes 0, 2 -> k-slots 2t, 2t+1; bytes 1, 3 ->
//     2t+8, 2t+9) and high nibbles likewise.  A nibble becomes fp16 1024 + q
//     by a mask-or (0x64006400), then one fp16 FMA applies the sub-block
//     scale and removes the bias: (1024 + q) sc - 1024 sc = q sc, exact
//     because the FMA rounds once and q sc is representable.  High nibbles
//     stay in place (1024 + 16 q) and take sc / 16 and -64 sc.
//   * B: lane 4T + t (T = 0, 1, 2: hi, mid, lo) holds term T of the x values
//     of the k-slots above; the other lanes hold zeros.  These fragments are
//     the same for every row, so each CTA builds them once per launch in
//     shared memory (6 bytes per element), indexed [super-block][word i]
//     [lane][MMA 2i, 2i+1] so a lane reads both of a word's fragments at once.
//   * C: thread t = 0 holds the hi and mid sums, t = 1 the lo sum (and a
//     zero column), t = 2, 3 zeros; the four lanes of a row are summed at
//     the end of the row group.
//
// Work split: each CTA owns rows [c0, c1) (balanced to one row), in row
// groups of 16 MT rows (clipped at matrix ends; MT = 2 MMA tiles per warp by
// default, which share each B fragment).  A row group is streamed in chunks
// of NW super-blocks (one per warp): one 3-D tensor copy (TMA, no multicast)
// of 16 MT rows x NW super-blocks per tile, or, for a short row group, one
// bulk copy per row.  Warp w takes super-block w of every chunk for all the
// group's rows; at the end of a row group the warps' partial sums meet in
// shared memory and warp 0 writes y.  A producer warp (its lane 0) fills the
// ring before the grid dependency wait and refills each stage once every
// compute warp has released it.  Rows longer than the activation fragments
// shared memory holds are done in parts of k, the rows' partial sums carried
// in shared memory and added in order.  All waits are bounded as in the
// other kernels.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "gemv.cuh"

namespace frc {

constexpr int kTc1Rows = 16;         // rows of one MMA tile (the MMA's M)
constexpr int kTc1MaxRows = 32;      // rows per row group, at most (two MMA tiles per warp)
constexpr int kTc1MaxWarps = 16;     // compute warps (one super-block each per chunk)
// compute warps of the widest two-tile instantiation: with the producer 12
// warps, three per SM sub-partition, which leaves each up to 170 registers
constexpr int kTc1MaxWarpsMt2 = 11;
constexpr int kTc1Lanes = 12;        // lanes of a B fragment that carry x terms
constexpr int kTc1FragBytes = 16 * kTc1Lanes * 8;  // per super-block: 16 MMAs x 12 lanes x 8 bytes
constexpr int kTc1ZeroBytes = 16 * kTc1Lanes * 8;  // the zero B fragment of lanes >= 12

// Shared-memory layout of gemv_tc1 (host and device).
struct Tc1Layout {
  int bars, red, scr, yacc, sums, invs, frags, zeros, stages, total;
};

__host__ __device__ constexpr int tc1_align(int v, int a) { return (v + a - 1) / a * a; }

// psb: super-blocks per part of k (the fragments held at a time); rows:
// the most rows one CTA owns (partial sums carried across parts); nbuf: 1,
// or 2 when a builder warp fills one fragment buffer while the compute warps
// read the other.
__host__ __device__ inline Tc1Layout tc1_layout(int nst, int psb, int rows, int stage_bytes, int nbuf = 1) {
  Tc1Layout L{};
  L.bars = 0;  // full[nst], empty[nst], frag_full[2], frag_empty[2], norm, then abort and void flags, inv norm
  L.red = tc1_align(16 * nst + 40 + 12, 16);         // [2][kTc1MaxWarps][row group] row partials
  L.scr = L.red + 2 * kTc1MaxWarps * kTc1MaxRows * 4;  // [kTc1MaxWarps] reduction scratch
  L.yacc = L.scr + kTc1MaxWarps * 4;                 // [rows] partial row sums over parts of k
  L.sums = tc1_align(L.yacc + rows * 4, 16);         // [nbuf][psb][8] fp32 sub-block sums of x
  L.invs = L.sums + nbuf * psb * 32;                 // [nbuf][psb] 1 / s per super-block
  L.frags = tc1_align(L.invs + nbuf * psb * 4, 128);  // [nbuf][psb][16][12] uint2
  L.zeros = L.frags + nbuf * psb * kTc1FragBytes;    // kTc1ZeroBytes of zeros
  L.stages = tc1_align(L.zeros + kTc1ZeroBytes, 128);
  L.total = L.stages + nst * stage_bytes;
  return L;
}

// Row stride of a stage: the chunk's bytes, dense (the layout a 3-D tensor
// copy of 16 rows x kc super-blocks lands in).
__host__ __device__ constexpr int tc1_row_stride(int kc, int ts) { return kc * ts; }

// Tensor maps per matrix of the launch: the matrix as a 3-D tensor of 8-byte
// words [rows][super-blocks][TS / 8] (strides row_bytes and TS bytes: 144
// for Q4_K, 176 for Q5_K), with boxes of kc super-blocks x TS / 8 words
// and 32, 16, 8, 4, 2 or 1 rows: a whole
// row group is one copy, a short one (a matrix or CTA end) one copy per set
// bit of its row count.
constexpr int kTc1Boxes = 6;  // rows 32 >> b for b < kTc1Boxes
struct Tc1Maps {
  CUtensorMap m[4][kTc1Boxes];
};

FRC_DEVICE_INLINE uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
FRC_DEVICE_INLINE uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
FRC_DEVICE_INLINE uint32_t hadd2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
FRC_DEVICE_INLINE uint32_t hmul2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
FRC_DEVICE_INLINE void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                     uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// d = a b (the accumulator starts at zero)
FRC_DEVICE_INLINE void mma_f16_16816_z(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}
// Shared-memory loads of data that TMA copies or other warps wrote before an
// mbarrier wait or a barrier: not volatile, but ordered after those waits by
// the memory clobber (the hardware schedule is the assembler's).
template <int OFF>
FRC_DEVICE_INLINE uint4 lds128f(uint32_t a) {
  uint4 v;
  asm("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4+%5];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "r"(a), "n"(OFF)
      : "memory");
  return v;
}
FRC_DEVICE_INLINE uint4 lds128u(uint32_t a) {
  uint4 v;
  asm("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}
FRC_DEVICE_INLINE uint2 lds64(uint32_t a) {
  uint2 v;
  asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a) : "memory");
  return v;
}
FRC_DEVICE_INLINE void sts64(uint32_t a, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}

// Thread-block clusters (split launches): every thread of the cluster
// arrives (release) and waits (acquire); shared memory of cluster rank
// `rank` at the address of a local shared variable.
FRC_DEVICE_INLINE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
FRC_DEVICE_INLINE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
FRC_DEVICE_INLINE uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(local), "r"(rank));
  return a;
}
FRC_DEVICE_INLINE float ld_cluster_f32(uint32_t a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}
FRC_DEVICE_INLINE uint32_t ld_cluster_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}

// fp16 constants, two per word
constexpr uint32_t kH2Bias = 0x64006400u;      // 1024, 1024 (with a nibble or byte in the mantissa)
constexpr uint32_t kH2Neg1024 = 0xE400E400u;   // -1024
constexpr uint32_t kH2Sixteenth = 0x2C002C00u; // 1/16
constexpr uint32_t kH2Neg64 = 0xD400D400u;     // -64

// The three fp16 terms of a and b (low and high halves of each word).
FRC_DEVICE_INLINE void split3(float a, float b, uint32_t& t0, uint32_t& t1, uint32_t& t2) {
  const __half2 h0 = __floats2half2_rn(a, b);
  const float2 f0 = __half22float2(h0);
  const float ra = a - f0.x, rb = b - f0.y;
  const __half2 h1 = __floats2half2_rn(ra, rb);
  const float2 f1 = __half22float2(h1);
  const __half2 h2 = __floats2half2_rn(ra - f1.x, rb - f1.y);
  t0 = *reinterpret_cast<const uint32_t*>(&h0);
  t1 = *reinterpret_cast<const uint32_t*>(&h1);
  t2 = *reinterpret_cast<const uint32_t*>(&h2);
}

// Power-of-two scale s with |m s| < 2^15 for the largest magnitude m of a
// super-block, and 1 / s.  The exponent is at least -113, its value for the
// largest finite fp32 m (so |m s| < 2^15 holds for every finite m and the
// fp16 terms never overflow), and at most 100: for m below 2^-86 the scale
// stays 2^100, so that d / s of a normal fp16 d stays a normal fp32 number
// (the terms then start below 2^14).
FRC_DEVICE_INLINE void tc1_scale(float m, float& s, float& inv) {
  int e = static_cast<int>((__float_as_uint(m) >> 23) & 0xFFu) - 127;  // floor(log2 m) for normal m
  int se = 14 - e;
  se = se < -113 ? -113 : (se > 100 ? 100 : se);
  s = __uint_as_float(static_cast<uint32_t>(127 + se) << 23);
  inv = __uint_as_float(static_cast<uint32_t>(127 - se) << 23);
}

// Q4_K scale and min bytes of sub-blocks 2t and 2t+1 from a block header
// (h.y = scales[0..3], h.z = scales[4..7], h.w = scales[8..11]): byte 0 of
// the results is sub-block 2t, byte 1 sub-block 2t+1.  sh = 16 (t & 1);
// lanes t >= 2 take the split 4+2-bit form (ggml's get_scale_min_k4).
FRC_DEVICE_INLINE void tc1_q4k_scales(const uint4& h, uint32_t sh, bool hi_t, uint32_t m1, uint32_t m2, uint32_t& sc,
                                      uint32_t& mn) {
  const uint32_t a = h.y >> sh, b = h.z >> sh, c = h.w >> sh;
  const uint32_t x1 = hi_t ? c : a;
  const uint32_t x2 = hi_t ? (c >> 4) : b;
  sc = (x1 & m1) | ((a >> 2) & m2);
  mn = (x2 & m1) | ((b >> 2) & m2);
}

// One super-block of MT 16-row MMA tiles for this warp (rows g + 16 m and
// g + 8 + 16 m of the row group, m < MT; the tiles share the B fragments).
// row: shared address of row g's block; xf: shared address of this lane's
// B fragment words for the super-block (lanes >= 12 point at a zero
// fragment), fragments 2i and 2i + 1 at xf + 192 i; sums: the super-block's
// 8 sub-block sums.  acc[2m], acc[2m+1] (rows g + 16 m, g + 8 + 16 m) gain
// d / s times the column sums; mn[...] gain dmin times the min terms.
//
// Q5_K (gguf.py:223-263) has the Q4_K header and nibbles (at byte 48) plus
// qh[32] at byte 16, whose bit 2t (2t + 1) of byte i is the fifth bit of
// element i of sub-block 2t (2t + 1).  The bit joins the fp16 lane below the
// bias: at bit 4 beside a low nibble (1024 + q), at bit 8 beside a high
// nibble (1024 + 16 q), so the same HFMA2 gives q sc exactly (q sc <= 31 x
// 63 = 1953; the fused product-add rounds once, at the exact result).
template <int Q, int MT>
FRC_DEVICE_INLINE void tc1_sb(uint32_t row, uint32_t stride, uint32_t xf, uint32_t sums, float inv_s, int t,
                                  uint32_t sh, bool hi_t, uint32_t m1, uint32_t m2, uint32_t bias, float (&acc)[2 * MT],
                                  float (&mn)[2 * MT]) {
  constexpr int R = 2 * MT;  // rows of this thread
  constexpr bool Q5 = Q == kQ5_K;
  constexpr uint32_t kQsOff = Q5 ? 48u : 16u;
  uint4 hd[R];
  uint32_t q[R], sl[R], nl[R], sg[R], ng[R], mw[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint32_t ra = row + static_cast<uint32_t>(8 * r) * stride;  // rows g, g + 8, g + 16, g + 24
    hd[r] = lds128f<0>(ra);
    q[r] = ra + kQsOff + 32u * static_cast<uint32_t>(t);
    uint32_t sc;
    tc1_q4k_scales(hd[r], sh, hi_t, m1, m2, sc, mw[r]);
    // (sc, sc) of the low sub-block, and (sc/16, sc/16) of the high one,
    // with their bias terms -1024 sc and -64 sc
    sl[r] = hadd2_u(prmt(sc, kH2Bias, 0x7050), kH2Neg1024);
    nl[r] = hmul2_u(sl[r], kH2Neg1024);
    sg[r] = hfma2_u(prmt(sc, kH2Bias, 0x7151), kH2Sixteenth, kH2Neg64);
    ng[r] = hmul2_u(sg[r], kH2Neg1024);
  }
  // per tile one accumulator over the super-block's 16 MMAs (the first
  // starts it at zero): low nibbles (sub-block 2t) and high nibbles (2t + 1)
  float c[MT][4];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    // words 4 half .. 4 half + 3 of chunk t in each row
    uint32_t w[R][4], hq[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint4 a = half ? lds128f<16>(q[r]) : lds128f<0>(q[r]);
      w[r][0] = a.x;
      w[r][1] = a.y;
      w[r][2] = a.z;
      w[r][3] = a.w;
      if constexpr (Q5) {
        // qh bytes 16 half .. 16 half + 15 (row start + 16), bits of
        // sub-blocks 2t, 2t + 1 moved to bits 0 and 1 of each byte
        const uint32_t qa = q[r] - kQsOff - 32u * static_cast<uint32_t>(t) + 16u;
        const uint4 b = half ? lds128f<16>(qa) : lds128f<0>(qa);
        hq[r][0] = b.x >> (2 * t);
        hq[r][1] = b.y >> (2 * t);
        hq[r][2] = b.z >> (2 * t);
        hq[r][3] = b.w >> (2 * t);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * half + j;
      // B fragments of MMAs 2i (low) and 2i + 1 (high), side by side
      const uint4 b = lds128u(xf + static_cast<uint32_t>(i * kTc1Lanes * 16));
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const uint32_t x0 = w[2 * m][j], x8 = w[2 * m + 1][j];
        const uint32_t s0 = x0 >> 8, s8 = x8 >> 8;
        const int r0 = 2 * m, r8 = 2 * m + 1;
        // the bias of each lane pair, with Q5_K's fifth bits below it
        uint32_t bl0 = bias, bl8 = bias, bs0 = bias, bs8 = bias, hl0 = bias, hl8 = bias, hs0 = bias, hs8 = bias;
        if constexpr (Q5) {
          const uint32_t h0 = hq[r0][j], h8 = hq[r8][j];
          bl0 = ((h0 << 4) & 0x00100010u) | bias;  // bytes 0, 2: bit 0 -> bit 4
          bl8 = ((h8 << 4) & 0x00100010u) | bias;
          bs0 = ((h0 >> 4) & 0x00100010u) | bias;  // bytes 1, 3: bit 8 -> bit 4
          bs8 = ((h8 >> 4) & 0x00100010u) | bias;
          hl0 = ((h0 << 7) & 0x01000100u) | bias;  // bytes 0, 2: bit 1 -> bit 8
          hl8 = ((h8 << 7) & 0x01000100u) | bias;
          hs0 = ((h0 >> 1) & 0x01000100u) | bias;  // bytes 1, 3: bit 9 -> bit 8
          hs8 = ((h8 >> 1) & 0x01000100u) | bias;
        }
        const uint32_t l0 = hfma2_u((x0 & 0x000F000Fu) | bl0, sl[r0], nl[r0]);
        const uint32_t l1 = hfma2_u((x8 & 0x000F000Fu) | bl8, sl[r8], nl[r8]);
        const uint32_t l2 = hfma2_u((s0 & 0x000F000Fu) | bs0, sl[r0], nl[r0]);
        const uint32_t l3 = hfma2_u((s8 & 0x000F000Fu) | bs8, sl[r8], nl[r8]);
        if (i == 0) {
          mma_f16_16816_z(c[m], l0, l1, l2, l3, b.x, b.y);
        } else {
          mma_f16_16816(c[m], l0, l1, l2, l3, b.x, b.y);
        }
        mma_f16_16816(c[m], hfma2_u((x0 & 0x00F000F0u) | hl0, sg[r0], ng[r0]),
                      hfma2_u((x8 & 0x00F000F0u) | hl8, sg[r8], ng[r8]),
                      hfma2_u((s0 & 0x00F000F0u) | hs0, sg[r0], ng[r0]),
                      hfma2_u((s8 & 0x00F000F0u) | hs8, sg[r8], ng[r8]), b.z, b.w);
      }
    }
  }
  // mins of sub-blocks 2t and 2t+1 against their x sums
  const uint2 xsw = lds64(sums + 8u * static_cast<uint32_t>(t));
  const float xs0 = __uint_as_float(xsw.x), xs1 = __uint_as_float(xsw.y);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    // columns 2t, 2t+1 of rows g and g+8: (hi, mid) for t = 0, (lo, 0) for
    // t = 1, zeros beyond
    const float s_0 = c[m][0] + c[m][1];
    const float s_8 = c[m][2] + c[m][3];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = 2 * m + h;
      const float d = half_bits_to_float(hd[r].x), dm = half_bits_to_float(hd[r].x >> 16);
      acc[r] = fmaf(d * inv_s, h ? s_8 : s_0, acc[r]);
      mn[r] = fmaf(dm, fmaf(static_cast<float>(mw[r] & 0xFFu), xs0, static_cast<float>((mw[r] >> 8) & 0xFFu) * xs1),
                   mn[r]);
    }
  }
}

FRC_DEVICE_INLINE float ldsf(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}

// Activations of sub-block j (32 consecutive elements of x), with the
// SwiGLU applied when x_mul is set (silu(gate) * up as the reference forms
// it, qwen2.py:1690-1751).
FRC_DEVICE_INLINE void tc1_load_sub(const GemvParams& p, int j, float (&v)[32]) {
  const float4* src = reinterpret_cast<const float4*>(p.x + static_cast<int64_t>(j) * 32);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 f = __ldg(src + q);
    v[4 * q] = f.x;
    v[4 * q + 1] = f.y;
    v[4 * q + 2] = f.z;
    v[4 * q + 3] = f.w;
  }
  if (p.x_mul) {
    const float4* us = reinterpret_cast<const float4*>(p.x_mul + static_cast<int64_t>(j) * 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 u = __ldg(us + q);
      const float uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float g = v[4 * q + e];
        const float sg = 1.0f / (1.0f + expf(-g));
        v[4 * q + e] = (sg * g) * uu[e];
      }
    }
  }
}

// The producer's position in the CTA's tile sequence: parts of k outermost,
// then row groups of 16 rows, then the part's chunks.
struct Tc1Cursor {
  int64_t t0;  // first row of the current row group
  Tile T;      // the current row group (set when its first chunk is issued)
  int rows;
  int ch;      // next chunk (index over the whole row)
  int part;    // current part of k
};

template <int TS>
FRC_DEVICE_INLINE void tc1_issue(const GemvParams& p, const Tc1Maps& maps, Tc1Cursor& c, int64_t c0, int64_t c1,
                                 uint8_t* dst, uint64_t* bar) {
  const int pc = p.tc_part_chunks;
  if (c.ch == c.part * pc) {
    c.T = tile_at(p, c.t0, c1, p.tc_rg);
    c.rows = static_cast<int>(c.T.t1 - c.t0);
  }
  const int kc = p.tc_kc, sbs = p.k / 256;
  // the group's rows as tensor boxes of 32, 16, ..., 1 rows (the
  // super-blocks past the row's end read as zeros and are not used), each
  // landing on a 128-byte boundary of the stage as tensor copies require;
  // rows left after the first box that would not are copied one bulk copy
  // per row (16-byte aligned)
  const uint32_t box_bytes = static_cast<uint32_t>(kc * TS);
  const int nsb = (c.ch + 1) * kc <= sbs ? kc : sbs - c.ch * kc;
  const uint32_t cb = static_cast<uint32_t>(nsb) * TS;
  int r0 = 0;
  uint32_t tx = 0;
  int nbox = 0, boxes[kTc1Boxes], starts[kTc1Boxes];
  for (int b = 0; b < kTc1Boxes; ++b) {
    const int box = kTc1MaxRows >> b;
    if (c.rows - r0 >= box && (static_cast<uint32_t>(r0) * static_cast<uint32_t>(p.tc_stride)) % 128u == 0) {
      boxes[nbox] = b;
      starts[nbox++] = r0;
      tx += static_cast<uint32_t>(box) * box_bytes;
      r0 += box;
    }
  }
  tx += static_cast<uint32_t>(c.rows - r0) * cb;
  mbar_arrive_expect_tx(bar, tx);
  for (int i = 0; i < nbox; ++i) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(dst + starts[i] * p.tc_stride)), "l"(reinterpret_cast<uint64_t>(&maps.m[c.T.m][boxes[i]])),
        "r"(0), "r"(c.ch * kc), "r"(static_cast<int>(c.T.local) + starts[i]), "r"(smem_u32(bar))
        : "memory");
  }
  if (r0 < c.rows) {
    const uint8_t* src = p.mat_w[c.T.m] + static_cast<uint64_t>(c.T.local + r0) * p.row_bytes +
                         static_cast<uint64_t>(c.ch) * kc * TS;
    for (int r = r0; r < c.rows; ++r)
      bulk_g2s(dst + r * p.tc_stride, src + static_cast<uint64_t>(r - r0) * p.row_bytes, cb, bar);
  }
  const int part_end = (c.part + 1) * pc < p.tc_nchunk ? (c.part + 1) * pc : p.tc_nchunk;
  if (++c.ch == part_end) {  // the row group's share of this part is issued
    c.t0 = c.T.t1;
    if (c.t0 >= c1) {  // every row group: on to the next part
      ++c.part;
      c.t0 = c0;
    }
    c.ch = c.part * pc;
  }
}

// Activation fragments, sub-block sums and scales of super-blocks [sb0, sb1)
// into one buffer: thread `tid` of `nthreads` (whole warps) owns sub-blocks
// 8 sb0 + tid, + nthreads, ...; lanes 8a .. 8a+7 hold one super-block.
FRC_DEVICE_INLINE void tc1_build(const GemvParams& p, int sb0, int sb1, int tid, int nthreads, float inv_norm,
                                 uint32_t frag_base, float* sums, float* invs) {
  const int rounds = (8 * (sb1 - sb0) + nthreads - 1) / nthreads;
  for (int rr = 0; rr < rounds; ++rr) {
    const int j = 8 * sb0 + tid + rr * nthreads;
    float v[32];
    if (j < 8 * sb1) {
      tc1_load_sub(p, j, v);
      if (p.x_norm_w) {
        const float4* ws = reinterpret_cast<const float4*>(p.x_norm_w + static_cast<int64_t>(j) * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 gw = __ldg(ws + q);
          const float gg[4] = {gw.x, gw.y, gw.z, gw.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) v[4 * q + e] = (v[4 * q + e] * inv_norm) * gg[e];
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = 0.f;
    }
    float m = 0.f, xsum = 0.f;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      m = fmaxf(m, fabsf(v[e]));
      xsum += v[e];
    }
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 4));
    if (j < 8 * sb1) {
      float sc, inv;
      tc1_scale(m, sc, inv);
      const int lj = j - 8 * sb0, sb = lj >> 3, jj = lj & 7, tt = jj >> 1, h = jj & 1;
      sums[lj] = xsum;
      if (jj == 0) invs[sb] = inv;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t p0, p1, p2, q0, q1, q2;
        split3(v[4 * i] * sc, v[4 * i + 2] * sc, p0, p1, p2);
        split3(v[4 * i + 1] * sc, v[4 * i + 3] * sc, q0, q1, q2);
        const uint32_t a = frag_base + static_cast<uint32_t>(((sb * 8 + i) * kTc1Lanes + tt) * 16 + h * 8);
        sts64(a, p0, q0);
        sts64(a + 64u, p1, q1);
        sts64(a + 128u, p2, q2);
      }
    }
  }
}

// MAXW: the most compute warps a launch of this instantiation has (16, or 15
// so that the CTA's 16 warps get 128 registers each instead of 96).
// MT: 16-row MMA tiles per warp and super-block (a row group is 16 MT rows).
// NB: rows in several parts of k with NB builder warps (the last ones) that
// build part p + 1's fragments into the second buffer while the compute
// warps read part p's; 0: the compute warps build every part.
template <int Q, int MAXW, int MT, int NB>
__global__ void __launch_bounds__((MAXW + 1 + NB) * 32, 1) gemv_tc1(const __grid_constant__ Tc1Maps maps,
                                                                   GemvParams p) {
  static_assert(Q == kQ4_K || Q == kQ5_K, "gemv_tc1 covers Q4_K and Q5_K");
  constexpr int TS = Fmt<Q>::TS;
  static_assert(MT == 1 || MT == 2, "one or two MMA tiles per warp");
  constexpr int RG = kTc1Rows * MT;
  static_assert(MAXW <= kTc1MaxWarps, "reduction buffers hold kTc1MaxWarps warps");
  static_assert(NB >= 0 && NB <= 2, "up to two builder warps");
  constexpr bool BUILDER = NB > 0;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = static_cast<int>(blockDim.x >> 5) - 1 - NB;  // compute warps; then the producer, the builders
  const int nct = nw * 32;
  const int ct = threadIdx.x;
  const int nst = p.nstage;
  const int sbs = p.k / 256;
  const int stage_bytes = p.stage_stride;
  const int kc = p.tc_kc, nch = p.tc_nchunk, pc = p.tc_part_chunks;
  const int nparts = (nch + pc - 1) / pc;
  constexpr int NBUF = BUILDER ? 2 : 1;
  const int psb = pc * kc;
  const Tc1Layout L = tc1_layout(nst, psb, p.tc_rows_max, stage_bytes, NBUF);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + nst;
  uint64_t* frag_full = empty + nst;   // [2] a part's fragments are built (builder)
  uint64_t* frag_empty = frag_full + 2;  // [2] a buffer's part is done (compute warps)
  uint64_t* norm_ready = frag_empty + 2;  // the RMSNorm scale is in shared memory
  int* abort_flag = reinterpret_cast<int*>(norm_ready + 1);
  int* void_flag = abort_flag + 1;  // an earlier gather's wait ran out
  float* norm_scale = reinterpret_cast<float*>(void_flag + 1);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* scr = reinterpret_cast<float*>(smem + L.scr);
  float* yacc = reinterpret_cast<float*>(smem + L.yacc);
  float* sums = reinterpret_cast<float*>(smem + L.sums);
  float* invs = reinterpret_cast<float*>(smem + L.invs);
  uint8_t* stages = smem + L.stages;

  if (ct == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], static_cast<uint32_t>(nw));
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&frag_full[i], BUILDER ? 32u * NB : 1u);
      mbar_init(&frag_empty[i], static_cast<uint32_t>(nw));
    }
    mbar_init(norm_ready, 1);
    *abort_flag = 0;
    *void_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  volatile int* abort = abort_flag;

  // split launches: the cluster's CTAs share one row range, CTA r taking
  // part r of k (no builder warps); otherwise every part, in order
  const int split = p.tc_split;
  int64_t c0, c1;
  int pb = 0, pe = nparts;
  if (split > 1) {
    const int64_t ranges = gridDim.x / split, j = blockIdx.x / split;
    c0 = j * p.n / ranges;
    c1 = (j + 1) * p.n / ranges;
    pb = static_cast<int>(cluster_rank());
    pe = pb + 1;
  } else {
    cta_rows(p.n, c0, c1);
  }
  const int ch_lo = pb * pc, ch_hi = pe * pc < nch ? pe * pc : nch;
  const int ntiles = count_tiles(p, c0, c1, RG) * (ch_hi - ch_lo);

  if (warp == nw) {
    // the producer warp: the weights are never written by another kernel, so
    // it streams them before the previous kernel in the stream has finished
    // (programmatic dependent launch)
    griddep_launch_dependents();
    if (lane == 0) {
      Tc1Cursor cur{c0, Tile{}, 0, ch_lo, pb};
      int issued = 0;
      for (; issued < ntiles; ++issued) {
        const int si = issued % nst;
        if (issued >= nst && !wait_phase(&empty[si], static_cast<uint32_t>(issued / nst - 1) & 1u, abort)) {
          atomicOr(p.status, kStatusEmptyWaitTimeout);
          break;
        }
        tc1_issue<TS>(p, maps, cur, c0, c1, stages + si * stage_bytes, &full[si]);
      }
      // the last stage-full of copies must land before the CTA may exit
      int zero = 0;
      for (int i = issued > nst ? issued - nst : 0; i < issued; ++i) {
        if (!wait_phase(&full[i % nst], static_cast<uint32_t>(i / nst) & 1u, &zero))
          atomicOr(p.status, kStatusDrainTimeout);
      }
    }
    if (split > 1) {  // every thread of the cluster takes part in both cluster barriers
      cluster_sync();
      cluster_sync();
    }
    return;
  }
  if (BUILDER && warp > nw) {
    // the builder warps: parts 1, 2, ... into buffer part % 2, each once the
    // compute warps have released that buffer's previous part
    const int bt = (warp - nw - 1) * 32 + lane;
    griddep_wait();
    griddep_launch_dependents();
    // x is final (an earlier fused gather complete) and its RMSNorm scale
    // is known once the compute warps publish it
    if (!wait_phase(norm_ready, 0u, abort)) return;
    const float inv_norm = *reinterpret_cast<volatile float*>(norm_scale);
    for (int part = 1; part < nparts; ++part) {
      const int b = part & 1;
      if (part >= 2 && !wait_phase(&frag_empty[b], static_cast<uint32_t>((part - 2) >> 1) & 1u, abort)) return;
      const int sb0 = part * pc * kc, sb1 = (part + 1) * pc * kc < sbs ? (part + 1) * pc * kc : sbs;
      tc1_build(p, sb0, sb1, bt, 32 * NB, inv_norm, smem_u32(smem + L.frags) + static_cast<uint32_t>(b * psb * kTc1FragBytes),
                reinterpret_cast<float*>(smem + L.sums) + b * psb * 8, reinterpret_cast<float*>(smem + L.invs) + b * psb);
      mbar_arrive(&frag_full[b]);  // every builder thread: its stores are released
    }
    return;
  }
  griddep_wait();
  griddep_launch_dependents();
  int g_world = p.g_world;
  if (p.w_world > 1) {  // an earlier fused gather must be complete on every rank
    if (ct < p.w_world) {
      const uint32_t e = *p.w_epoch;
      const uint64_t t0 = global_ns();
      while (true) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.w_flags + ct) : "memory");
        if (static_cast<int32_t>(v - e) >= 0) break;
        if (global_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.status, kStatusGatherTimeout);
          *void_flag = 1;  // read after the barrier below
          break;
        }
      }
    }
    named_barrier_sync(1, nct);
    // after a gather wait that ran out a peer may still read its buffer:
    // keep the outputs local and publish nothing (the status bit tells the
    // caller the step is void)
    if (*reinterpret_cast<volatile int*>(void_flag)) g_world = 1;
  }

  const int nsub = p.k / 32;
  float inv_norm = 1.f;
  if (p.x_norm_w) {  // RMSNorm of the whole row of x (qwen2.py:365-378)
    float ss = 0.f;
    for (int j = ct; j < nsub; j += nct) {
      float v[32];
      tc1_load_sub(p, j, v);
#pragma unroll
      for (int e = 0; e < 32; ++e) ss = fmaf(v[e], v[e], ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) scr[warp] = ss;
    named_barrier_sync(1, nct);
    ss = 0.f;
    for (int w = 0; w < nw; ++w) ss += scr[w];
    inv_norm = 1.0f / sqrtf(ss / static_cast<float>(p.k) + p.x_norm_eps);
  }
  if (BUILDER && ct == 0) {  // the builder reads x and normalises the later parts with the same scale
    *norm_scale = inv_norm;
    mbar_arrive(norm_ready);
  }
  // the zero fragment read by lanes >= 12 (columns 3..7 of B)
  const uint32_t zero_base = smem_u32(smem + L.zeros);
  for (int i = ct; i < kTc1ZeroBytes / 8; i += nct) sts64(zero_base + 8u * i, 0u, 0u);

  const int g = lane >> 2, t = lane & 3;
  const bool hi_t = t >= 2;
  const uint32_t sh = static_cast<uint32_t>(t & 1) * 16u;
  const uint32_t m1 = hi_t ? 0x0F0Fu : 0x3F3Fu, m2 = hi_t ? 0x3030u : 0u;
  const uint32_t frag_base = smem_u32(smem + L.frags);
  // lanes < 12 read their fragment words (stride one super-block), the rest
  // the zero fragment (stride 0)
  const uint32_t xf_lane = lane < kTc1Lanes ? frag_base + static_cast<uint32_t>(lane) * 16u : zero_base;
  const uint32_t xf_step = lane < kTc1Lanes ? static_cast<uint32_t>(kTc1FragBytes) : 0u;
  const uint32_t stride = static_cast<uint32_t>(p.tc_stride);
  const uint32_t row_lane = smem_u32(stages) + static_cast<uint32_t>(g) * stride + static_cast<uint32_t>(warp) * TS;
  const uint32_t sums_s = smem_u32(sums), invs_s = smem_u32(invs);
  int s = 0;
  uint32_t ph = 0u;
  int par = 0;
  for (int part = pb; part < pe; ++part) {
    const int ch0 = part * pc, ch1 = (part + 1) * pc < nch ? (part + 1) * pc : nch;
    const int sb0 = ch0 * kc;
    const int b = BUILDER ? (part & 1) : 0;  // this part's fragment buffer
    bool frags_ok = true;
    if (!BUILDER || part == pb) {
      // x fragments of super-blocks [sb0, sb1), built by the compute warps
      // (without a builder the previous part's fragments are free: every
      // warp has passed the barrier that ended its last row group)
      const int sb1 = ch1 * kc < sbs ? ch1 * kc : sbs;
      tc1_build(p, sb0, sb1, ct, nct, inv_norm, frag_base, sums, invs);
      named_barrier_sync(1, nct);  // fragments, sums, scales (and zeros) complete
    } else {
      frags_ok = wait_phase(&frag_full[b], static_cast<uint32_t>((part - 1) >> 1) & 1u, abort);
    }
    const uint32_t boff = static_cast<uint32_t>(b * psb);
    const uint32_t xf_part = xf_lane + (lane < kTc1Lanes ? boff * static_cast<uint32_t>(kTc1FragBytes) : 0u);
    const uint32_t sums_part = sums_s + boff * 32u, invs_part = invs_s + boff * 4u;

    // ---- row groups over this part's chunks ------------------------------
    for (int64_t t0 = c0; t0 < c1;) {
      const Tile T = tile_at(p, t0, c1, RG);
      const int rows = static_cast<int>(T.t1 - t0);
      float acc[2 * MT], mn[2 * MT];
#pragma unroll
      for (int r = 0; r < 2 * MT; ++r) acc[r] = mn[r] = 0.f;
      // the row group's chunks with M MMA tiles per warp (a: 2 M row sums,
      // b: 2 M min terms)
      auto run_chunks = [&](auto& a, auto& b) {
        constexpr int M = std::extent<std::remove_reference_t<decltype(a)>>::value / 2;
        for (int ch = ch0; ch < ch1; ++ch) {
          const int sb = ch * kc + warp;  // this warp's super-block of the chunk
          if (wait_phase(&full[s], ph, abort)) {
            if (sb < sbs && frags_ok) {
              const uint32_t lsb = static_cast<uint32_t>(sb - sb0);
              tc1_sb<Q, M>(row_lane + static_cast<uint32_t>(s * stage_bytes), stride, xf_part + lsb * xf_step,
                           sums_part + lsb * 32u, ldsf(invs_part + 4u * lsb), t, sh, hi_t, m1, m2, p.tc_bias, a, b);
            }
          } else if (lane == 0) {
            atomicOr(p.status, kStatusFullWaitTimeout);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
          if (++s == nst) {
            s = 0;
            ph ^= 1u;
          }
        }
      };
      // a row group of at most 16 rows (the short last group of a CTA or a
      // matrix) converts and multiplies its first MMA tile only: half the
      // work of a full group (Llama-3-70B gate+up: each CTA's 388 rows are
      // 12 groups of 32 and one of 4)
      bool one_tile = false;
      if constexpr (MT == 2) one_tile = rows <= kTc1Rows;
      if (one_tile) {
        float a1[2] = {0.f, 0.f}, b1[2] = {0.f, 0.f};
        run_chunks(a1, b1);
        acc[0] = a1[0];
        acc[1] = a1[1];
        mn[0] = b1[0];
        mn[1] = b1[1];
      } else {
        run_chunks(acc, mn);
      }
      // rows g + 8 r: the four lanes t of a row, then the warps
      float* rb = red + par * kTc1MaxWarps * RG;
#pragma unroll
      for (int r = 0; r < 2 * MT; ++r) {
        float v = acc[r] - mn[r];
        v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
        v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
        if (t == 0) rb[warp * RG + g + 8 * r] = v;
      }
      named_barrier_sync(1, nct);
      if (warp == 0) {
        // RG = 16: lane l adds the partials of row l & 15 from warps
        // 8 (l >> 4) .. 8 (l >> 4) + 7, then the two halves meet; RG = 32:
        // lane l adds row l's partials from every warp.  Independent loads,
        // the same order for every row and every launch.
        float h = 0.f;
        if constexpr (RG == 16) {
          const int r = lane & 15, w0 = 8 * (lane >> 4);
#pragma unroll
          for (int w = 0; w < 8; ++w) h += w0 + w < nw ? rb[(w0 + w) * RG + r] : 0.f;
          h += __shfl_xor_sync(0xFFFFFFFFu, h, 16);
        } else {
#pragma unroll
          for (int w = 0; w < MAXW; ++w) h += w < nw ? rb[w * RG + lane] : 0.f;
        }
        if (lane < rows) {
          // parts of k are added in order: ((part 0 + part 1) + part 2) ...
          // (a split launch keeps its part's sums for cluster rank 0)
          float y = h;
          float* ya = yacc + (t0 - c0) + lane;
          if (part > pb) y = *ya + y;
          if (part + 1 < pe || split > 1) {
            *ya = y;
          } else if (!*abort) {
            put_y(p, g_world, p.mat_y[T.m] + T.local + lane, y);
          }
        }
      }
      par ^= 1;
      t0 = T.t1;
    }
    // every compute warp has passed the last row group's barrier: this
    // part's buffer is free for the builder's part + 2
    if (BUILDER && part + 2 < nparts && lane == 0) mbar_arrive(&frag_empty[b]);
  }
  if (split > 1) {
    // every CTA's part sums are in its shared memory: rank 0 adds them in
    // part order, as the one-CTA launch does, and writes y (none if a wait
    // ran out in any CTA of the cluster); the second barrier keeps the
    // others' shared memory until rank 0 has read it
    cluster_sync();
    if (pb == 0) {
      bool bad = *abort != 0;
      for (int r = 1; r < split; ++r)
        bad = bad || ld_cluster_u32(cluster_addr(smem_u32(abort_flag), static_cast<uint32_t>(r))) != 0u;
      if (!bad) {
        for (int i = ct; i < static_cast<int>(c1 - c0); i += nct) {
          float y = yacc[i];
          const uint32_t la = smem_u32(yacc + i);
          for (int r = 1; r < split; ++r) y = y + ld_cluster_f32(cluster_addr(la, static_cast<uint32_t>(r)));
          const int64_t row = c0 + i;
          int m = 0;
          while (m + 1 < p.nmat && row >= p.mat_end[m]) ++m;
          put_y(p, g_world, p.mat_y[m] + (row - (m ? p.mat_end[m - 1] : 0)), y);
        }
      }
    }
    cluster_sync();
  }
  if (g_world > 1) {  // publish this CTA's gathered rows
    named_barrier_sync(1, nct);
    if (ct == 0) gather_arrive(p, g_world, 1);
  }
}

}  // namespace frc
