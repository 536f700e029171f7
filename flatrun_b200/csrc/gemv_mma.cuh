// Batched GEMV (2..16 activation columns) on the integer tensor cores.
//
// Pre-pass (mma_quantise_x): every activation column is cut into 32-element
// groups; each group gets one fp32 scale sx and 16-bit integers
// xq = rint(x / sx) (|xq| <= 32639, the grid of the batch-1 kernel), split into
// two signed byte planes xq = 256 xh + xl.  The records are written to scratch
// memory chunk-major: for every k-chunk of kMmaKC elements, every column's
// record holds the h plane, the l plane (words permuted so a thread's two
// fragment words are adjacent) and per group 32 bytes of sums:
// (sx, sx*sum(xq), then for each 16-element half -32*sum(xh), -32*sum(xl)).
//
// Main kernel (gemv_mma): persistent CTAs own contiguous rows, processed in
// row blocks of 16*MT rows.  One producer thread streams, per (row block,
// chunk), the block's chunk bytes as 2-D tensor boxes (the matrix viewed as
// rows of G consecutive matrix rows, G * row_bytes a multiple of 16: one box
// of R = 16*MT/G tensor rows per row residue) and the chunk's activation
// records (one bulk copy) into a ring of shared-memory stages.  Eight
// consumer warps split each chunk's k-steps, two 32-element steps (Q6_K: four
// 16-element steps) per warp chosen so the warp's steps share their quant
// bytes; for every step and 16-row tile they run mma.sync m16n8k32 (m16n8k16 for Q6_K's 16-element scale
// groups) with the raw quant values as A (Q4_K: one mask per word) and the x
// byte planes as B: columns 2c and 2c+1 of an 8-wide N tile are the h and l
// planes of activation column c, so a thread's accumulator pair combines to
// T = 256 c0 + c1 = sum(q * xq) (accumulators seeded so each plane's sum
// reads back as a float after one add).  Each (row, step, column) then adds
// sx * (ds * T - dm * X) in fp32, with (ds, dm) from a per-warp shared table
// (K-quants: d*sc and dmin*m; Q8_0: d and 0; Q1_0, whose bits enter as +1/-1
// bytes: d and 0; Q6_K: d*sc, its -32 offset folded into the seeds).  At the
// end of a row block the warps' partial sums are reduced through shared
// memory and written to y.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "gemv.cuh"

namespace frc {

constexpr int kMmaKC = 512;                                     // k elements per chunk
constexpr int kMmaPlane = kMmaKC + 32;                          // bytes per byte plane (padded)
constexpr int kMmaMeta = 32;                                    // bytes of sums per 32-element group
constexpr int kMmaColBytes = 2 * kMmaPlane + (kMmaKC / 32) * kMmaMeta;  // 1600: per column per chunk
// Accumulator seed: the int32 bits of 1.5 * 2^23.  An MMA started from it
// leaves bits that read as the float 1.5 * 2^23 + sum for |sum| < 2^22, so one
// FADD recovers each plane's exact integer sum (no int->float conversion).
constexpr int kMagicBits = 0x4B400000;
constexpr float kMagicF = 12582912.0f;
constexpr int kMmaWarps = 8;                                    // consumer warps

struct MmaParams {
  const uint8_t* w;
  float* y;           // (batch, n)
  int64_t n;
  int k;
  int batch;
  int row_bytes;
  int chunk_bytes;    // bytes of a full chunk of one row
  int nchunk;
  int ncols;          // 4 * NG (records per chunk)
  const uint8_t* xrec;
  // weight tiles: the matrix is read as a 2-D tensor whose rows are groups of
  // G matrix rows (G * row_bytes is a multiple of 16); a row block of RM rows
  // is G boxes (one per row residue j) of R = RM / G tensor rows x W bytes
  int G, R, W;
  int logG, logR;     // G = 1 << logG, R = 1 << logR
  int JS;             // shared-memory bytes between the boxes of a stage
  int64_t n_full;     // rows covered by whole tensor rows (G * floor(n / G))
  int WT;             // per-row slot of the < G rows past n_full (1-D copies)
  int tail_off;       // stage offset of those slots
  int x_off;          // stage offset of the activation records
  int stage_stride;
  int nstage;
  uint32_t* status;
};

// ---------------------------------------------------------------------------
// activation pre-pass: one thread per (chunk, column, 32-element group)
// ---------------------------------------------------------------------------
static __global__ void __launch_bounds__(256) mma_quantise_x(const float* __restrict__ x, int k, int batch, int ncols,
                                                      int nchunk, uint8_t* __restrict__ xrec) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" :::);
  constexpr int G = kMmaKC / 32;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(nchunk) * ncols * G;
  if (tid >= total) return;
  const int gi = static_cast<int>(tid % G);
  const int col = static_cast<int>((tid / G) % ncols);
  const int ch = static_cast<int>(tid / (static_cast<int64_t>(G) * ncols));
  const int e0 = ch * kMmaKC + gi * 32;
  float v[32];
  if (col < batch && e0 < k) {  // k is a multiple of 32: a group is all in or all out
    const float4* s4 = reinterpret_cast<const float4*>(x + static_cast<int64_t>(col) * k + e0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 t = __ldg(s4 + i);
      v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float sx = amax > 0.f ? amax / static_cast<float>(kXqMax) : 1.0f;
  const float inv = amax > 0.f ? static_cast<float>(kXqMax) / amax : 0.0f;
  uint32_t hw[8], lw[8];
  int ssum = 0, sh[2] = {0, 0}, sl[2] = {0, 0};
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    uint32_t h = 0, l = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      int q = round_to_int(v[4 * w + b], inv);
      q = q > kXqMax ? kXqMax : (q < -kXqMax ? -kXqMax : q);
      const int qh = (q + 128) >> 8;
      const int ql = q - 256 * qh;
      ssum += q;
      sh[w >> 2] += qh;
      sl[w >> 2] += ql;
      h |= (static_cast<uint32_t>(qh) & 0xFFu) << (8 * b);
      l |= (static_cast<uint32_t>(ql) & 0xFFu) << (8 * b);
    }
    hw[w] = h;
    lw[w] = l;
  }
  uint8_t* rec = xrec + (static_cast<int64_t>(ch) * ncols + col) * kMmaColBytes;
  // words permuted [0,4,1,5,2,6,3,7]: fragment words t and t+4 are adjacent
  uint4* ph = reinterpret_cast<uint4*>(rec + gi * 32);
  uint4* pl = reinterpret_cast<uint4*>(rec + kMmaPlane + gi * 32);
  ph[0] = make_uint4(hw[0], hw[4], hw[1], hw[5]);
  ph[1] = make_uint4(hw[2], hw[6], hw[3], hw[7]);
  pl[0] = make_uint4(lw[0], lw[4], lw[1], lw[5]);
  pl[1] = make_uint4(lw[2], lw[6], lw[3], lw[7]);
  uint4* pm = reinterpret_cast<uint4*>(rec + 2 * kMmaPlane + gi * kMmaMeta);
  pm[0] = make_uint4(__float_as_uint(sx), __float_as_uint(sx * static_cast<float>(ssum)),
                     static_cast<uint32_t>(-32 * sh[0]), static_cast<uint32_t>(-32 * sl[0]));
  pm[1] = make_uint4(static_cast<uint32_t>(-32 * sh[1]), static_cast<uint32_t>(-32 * sl[1]), 0u, 0u);
}

// ---------------------------------------------------------------------------
// tensor-core fragments and the copy path
// ---------------------------------------------------------------------------
template <bool AU8>
FRC_DEVICE_INLINE void mma_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                               uint32_t b1) {
  if constexpr (AU8) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

FRC_DEVICE_INLINE void mma_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
               : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
               : "r"(a0), "r"(a1), "r"(b0));
}

FRC_DEVICE_INLINE uint32_t ld32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Four bytes at a 2-byte aligned shared-memory address, as two 16-bit loads
// and one byte permute (no branch on the alignment: rows of one warp differ).
FRC_DEVICE_INLINE uint32_t ld32_h2(const uint8_t* p) {
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
  return __byte_perm(static_cast<uint32_t>(q[0]), static_cast<uint32_t>(q[1]), 0x5410);
}

// Spread bits 0..3 of `nib` to bit 0 of bytes 0..3.
FRC_DEVICE_INLINE uint32_t spread4(uint32_t nib) { return ((nib & 0xFu) * 0x00204081u) & 0x01010101u; }

// ---------------------------------------------------------------------------
// Per-format work of consumer warp w (of kMmaWarps) on one 512-element chunk
// of a row.  The warp owns SPW steps of KSTEP elements:
//   elem(w, j)          first element of step j inside the chunk
//   xgroup(w, j)        the step's 32-element activation group
//   xhalf(w)            KSTEP 16: which half of that group (warp-constant)
//   scales(row, w, ds, dm)  per step: y += sx * (ds * T - dm * X); dm only
//                       for formats with mins (HAS_MIN)
//   decode(row, w, t, lo, hi)  this thread's A-fragment words per step:
//                       elements 4t..4t+3 (lo) and 16+4t..16+4t+3 (hi)
// `row` points at the row's chunk in shared memory (2-byte aligned; 16-byte
// aligned for Q4_K/Q5_K, whose rows are whole 16-byte multiples).
// ---------------------------------------------------------------------------
template <int Q> struct Mm;

// Q4_K: warp w -> block w/4, sub-block pair p = w%4 (low and high nibbles of
// the same 32 bytes).  High nibbles enter the MMA as q*16 (unsigned A, mask
// 0xF0), compensated by ds/16.
template <> struct Mm<kQ4_K> {
  static constexpr int KSTEP = 32, SPW = 2;
  static constexpr bool AU8 = true;
  static FRC_DEVICE_INLINE int elem(int w, int j) { return 32 * (2 * w + j); }
  static FRC_DEVICE_INLINE int xgroup(int w, int j) { return 2 * w + j; }
  static FRC_DEVICE_INLINE int xhalf(int) { return 0; }
  static constexpr bool HAS_MIN = true;
  static FRC_DEVICE_INLINE void scales(const uint8_t* row, int w, float (&ds)[SPW], float (&dm)[SPW]) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(row + 144 * (w >> 2));
    const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
    float sc0, m0, sc1, m1;
    scale_min_k4_words(2 * (w & 3), hdr.y, hdr.z, hdr.w, sc0, m0);
    scale_min_k4_words(2 * (w & 3) + 1, hdr.y, hdr.z, hdr.w, sc1, m1);
    ds[0] = d * sc0;
    dm[0] = dmin * m0;
    ds[1] = d * sc1 * 0.0625f;
    dm[1] = dmin * m1;
  }
  static FRC_DEVICE_INLINE void decode(const uint8_t* row, int w, int t, uint32_t (&lo)[SPW], uint32_t (&hi)[SPW]) {
    const uint8_t* qs = row + 144 * (w >> 2) + 16 + 32 * (w & 3) + 4 * t;
    const uint32_t a = ld32(qs), b = ld32(qs + 16);
    lo[0] = a & 0x0F0F0F0Fu;
    hi[0] = b & 0x0F0F0F0Fu;
    lo[1] = a & 0xF0F0F0F0u;
    hi[1] = b & 0xF0F0F0F0u;
  }
};

// Q5_K: as Q4_K, the fifth bit from qh (bit sb of byte l).
template <> struct Mm<kQ5_K> {
  static constexpr int KSTEP = 32, SPW = 2;
  static constexpr bool AU8 = false;
  static FRC_DEVICE_INLINE int elem(int w, int j) { return 32 * (2 * w + j); }
  static FRC_DEVICE_INLINE int xgroup(int w, int j) { return 2 * w + j; }
  static FRC_DEVICE_INLINE int xhalf(int) { return 0; }
  static constexpr bool HAS_MIN = true;
  static FRC_DEVICE_INLINE void scales(const uint8_t* row, int w, float (&ds)[SPW], float (&dm)[SPW]) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(row + 176 * (w >> 2));
    const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
    float sc0, m0, sc1, m1;
    scale_min_k4_words(2 * (w & 3), hdr.y, hdr.z, hdr.w, sc0, m0);
    scale_min_k4_words(2 * (w & 3) + 1, hdr.y, hdr.z, hdr.w, sc1, m1);
    ds[0] = d * sc0;
    dm[0] = dmin * m0;
    ds[1] = d * sc1;
    dm[1] = dmin * m1;
  }
  static FRC_DEVICE_INLINE void decode(const uint8_t* row, int w, int t, uint32_t (&lo)[SPW], uint32_t (&hi)[SPW]) {
    const uint8_t* blk = row + 176 * (w >> 2);
    const int p = w & 3;
    const uint32_t a = ld32(blk + 48 + 32 * p + 4 * t), b = ld32(blk + 64 + 32 * p + 4 * t);
    // bit sb of every qh byte moved to bit 4 of that byte
    const uint32_t ha = ld32(blk + 16 + 4 * t), hb = ld32(blk + 32 + 4 * t);
    const int s0 = 2 * p, s1 = 2 * p + 1;
    lo[0] = (a & 0x0F0F0F0Fu) | (((ha >> s0) << 4) & 0x10101010u);
    hi[0] = (b & 0x0F0F0F0Fu) | (((hb >> s0) << 4) & 0x10101010u);
    lo[1] = ((a >> 4) & 0x0F0F0F0Fu) | (((ha >> s1) << 4) & 0x10101010u);
    hi[1] = ((b >> 4) & 0x0F0F0F0Fu) | (((hb >> s1) << 4) & 0x10101010u);
  }
};

// Q8_0: warp w -> blocks 2w, 2w+1.
template <> struct Mm<kQ8_0> {
  static constexpr int KSTEP = 32, SPW = 2;
  static constexpr bool AU8 = false;
  static FRC_DEVICE_INLINE int elem(int w, int j) { return 32 * (2 * w + j); }
  static FRC_DEVICE_INLINE int xgroup(int w, int j) { return 2 * w + j; }
  static FRC_DEVICE_INLINE int xhalf(int) { return 0; }
  static constexpr bool HAS_MIN = false;
  static FRC_DEVICE_INLINE void scales(const uint8_t* row, int w, float (&ds)[SPW], float (&)[SPW]) {
#pragma unroll
    for (int j = 0; j < SPW; ++j) ds[j] = half_bits_to_float(ld_u16(row + 34 * (2 * w + j)));
  }
  static FRC_DEVICE_INLINE void decode(const uint8_t* row, int w, int t, uint32_t (&lo)[SPW], uint32_t (&hi)[SPW]) {
#pragma unroll
    for (int j = 0; j < SPW; ++j) {
      const uint8_t* qs = row + 34 * (2 * w + j) + 2 + 4 * t;
      lo[j] = ld32_h2(qs);
      hi[j] = ld32_h2(qs + 16);
    }
  }
};

// Q1_0: warp w -> block w/2, 32-element steps 2(w%2), 2(w%2)+1; bits enter the
// MMA as +1 / -1 bytes (~(bit * 0xFE)), so ds = d and there is no offset.
template <> struct Mm<kQ1_0> {
  static constexpr int KSTEP = 32, SPW = 2;
  static constexpr bool AU8 = false;
  static FRC_DEVICE_INLINE int elem(int w, int j) { return 128 * (w >> 1) + 32 * (2 * (w & 1) + j); }
  static FRC_DEVICE_INLINE int xgroup(int w, int j) { return 4 * (w >> 1) + 2 * (w & 1) + j; }
  static FRC_DEVICE_INLINE int xhalf(int) { return 0; }
  static constexpr bool HAS_MIN = false;
  static FRC_DEVICE_INLINE void scales(const uint8_t* row, int w, float (&ds)[SPW], float (&)[SPW]) {
    const float d = half_bits_to_float(ld_u16(row + 18 * (w >> 1)));
#pragma unroll
    for (int j = 0; j < SPW; ++j) ds[j] = d;
  }
  static FRC_DEVICE_INLINE void decode(const uint8_t* row, int w, int t, uint32_t (&lo)[SPW], uint32_t (&hi)[SPW]) {
    const uint8_t* bits = row + 18 * (w >> 1) + 2 + 8 * (w & 1);
#pragma unroll
    for (int j = 0; j < SPW; ++j) {
      const uint32_t v = ld32_h2(bits + 4 * j);
      lo[j] = ~(spread4(v >> (4 * t)) * 0xFEu);
      hi[j] = ~(spread4(v >> (4 * t + 16)) * 0xFEu);
    }
  }
};

// Q6_K: 16-element steps.  Warp w -> block b = w/4, half h = (w/2)%2 and
// 16-element half lh = w%2 of all four 32-element quarters r = j: quarters
// 0/2 share the low/high nibbles of one ql word, 1/3 of another, and all four
// share the qh word (2 bits each).
template <> struct Mm<kQ6_K> {
  static constexpr int KSTEP = 16, SPW = 4;
  static constexpr bool AU8 = false;
  static FRC_DEVICE_INLINE int elem(int w, int j) { return 256 * (w >> 2) + 128 * ((w >> 1) & 1) + 32 * j + 16 * (w & 1); }
  static FRC_DEVICE_INLINE int xgroup(int w, int j) { return 8 * (w >> 2) + 4 * ((w >> 1) & 1) + j; }
  static FRC_DEVICE_INLINE int xhalf(int w) { return w & 1; }
  static constexpr bool HAS_MIN = false;
  static FRC_DEVICE_INLINE void scales(const uint8_t* row, int w, float (&ds)[SPW], float (&)[SPW]) {
    const uint8_t* blk = row + 210 * (w >> 2);
    const float d = half_bits_to_float(ld_u16(blk + 208));
    uint32_t sw[2];
    lds_words_a2<2>(blk + 192 + 8 * ((w >> 1) & 1), sw);  // scales[8h .. 8h+7]
#pragma unroll
    for (int j = 0; j < SPW; ++j) {
      const int byte = 2 * j + (w & 1);  // scales[8h + 2r + lh]
      const int sc = static_cast<int>(static_cast<int8_t>((sw[byte >> 2] >> (8 * (byte & 3))) & 0xFFu));
      ds[j] = d * static_cast<float>(sc);
    }
  }
  static FRC_DEVICE_INLINE void decode(const uint8_t* row, int w, int t, uint32_t (&lo)[SPW], uint32_t (&hi)[SPW]) {
    const int h = (w >> 1) & 1, lh = w & 1;
    const uint8_t* blk = row + 210 * (w >> 2);
    const uint32_t ql0 = ld32_h2(blk + 64 * h + 16 * lh + 4 * t);
    const uint32_t ql1 = ld32_h2(blk + 64 * h + 32 + 16 * lh + 4 * t);
    const uint32_t qh = ld32_h2(blk + 128 + 32 * h + 16 * lh + 4 * t);
    // bits 2r, 2r+1 of every qh byte moved to bits 4, 5 of that byte
    lo[0] = (ql0 & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
    lo[1] = (ql1 & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
    lo[2] = ((ql0 >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
    lo[3] = ((ql1 >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
#pragma unroll
    for (int j = 0; j < SPW; ++j) hi[j] = 0u;
  }
};

// 2-D tensor copy of one box into shared memory, completion on `bar`
// (coordinates: x in 8-byte elements, always even; y in tensor rows).
FRC_DEVICE_INLINE void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Row-block slot L (0 .. RM-1) -> matrix row: box j = L / R, tensor row i = L % R.
FRC_DEVICE_INLINE int64_t slot_row(const MmaParams& p, int64_t row0, int L) {
  return row0 + (static_cast<int64_t>(L & (p.R - 1)) << p.logG) + (L >> p.logR);
}

// Stage-relative slot of row-block slot L (matrix row q), without the
// chunk's 16-byte phase (q * row_bytes + choff) % 16.  Rows of a box share
// that phase.  The < G rows in [n_full, n) have their own slots; slots of
// rows past n (padding of the last row block, computed and discarded) stay
// in the boxes.
FRC_DEVICE_INLINE int slot_offset(const MmaParams& p, int64_t q, int L) {
  if (q >= p.n_full && q < p.n) return p.tail_off + static_cast<int>(q - p.n_full) * p.WT;
  return (L >> p.logR) * p.JS + (L & (p.R - 1)) * p.W;
}

// Shared memory: [mbarriers | abort] 256 B, reduction [W][RM][NC] floats,
// per-warp scale tables [SPW][RM] of ds (float) or, for formats with mins,
// (ds, dm) (float2), step-major so a warp's lanes touch consecutive words;
// rounded to 128 B; then the stages.
template <int Q, int NG, int MT>
__host__ __device__ constexpr int mma_header_bytes() {
  return (256 + kMmaWarps * 16 * MT * 4 * NG * 4 + kMmaWarps * 16 * MT * Mm<Q>::SPW * 4 * (Mm<Q>::HAS_MIN ? 2 : 1) +
          127) / 128 * 128;
}

template <int Q, int NG, int MT>
__global__ void __launch_bounds__((kMmaWarps + 1) * 32, 1)
    gemv_mma(const __grid_constant__ CUtensorMap tmap, MmaParams p) {
  using F = Fmt<Q>;
  using M = Mm<Q>;
  constexpr int RM = 16 * MT, NC = 4 * NG, SPW = M::SPW;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + p.nstage;
  int* abort_flag = reinterpret_cast<int*>(empty + p.nstage);
  float* red = reinterpret_cast<float*>(smem + 256);
  constexpr int TABW = SPW * RM * (M::HAS_MIN ? 2 : 1);  // floats per warp
  float* tab_all = reinterpret_cast<float*>(smem + 256 + kMmaWarps * RM * NC * 4);
  using TabT = typename std::conditional<M::HAS_MIN, float2, float>::type;
  uint8_t* stages = smem + mma_header_bytes<Q, NG, MT>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  if (smem_u32(smem) & 127u) {  // tensor copies need 128-byte aligned boxes
    if (threadIdx.x == 0) atomicOr(p.status, kStatusSmemMisaligned);
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nstage; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMmaWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // rows of this CTA: whole G-row groups
  const int64_t ngrp = (p.n + p.G - 1) >> p.logG;
  const int64_t r0 = (static_cast<int64_t>(blockIdx.x) * ngrp / gridDim.x) << p.logG;
  int64_t r1 = (static_cast<int64_t>(blockIdx.x + 1) * ngrp / gridDim.x) << p.logG;
  if (r1 > p.n) r1 = p.n;
  const int nrb = static_cast<int>((r1 - r0 + RM - 1) / RM);
  const int items = nrb * p.nchunk;
  volatile int* abort = abort_flag;
  const uint64_t wtot = static_cast<uint64_t>(p.n) * p.row_bytes;
  const int xbytes = NC * kMmaColBytes;
  // bytes of the last (possibly partial) chunk of a row
  const int ce_last = p.k - (p.nchunk - 1) * kMmaKC;
  const uint64_t cb_last = static_cast<uint64_t>(ce_last / F::QK * F::TS);

  if (warp == kMmaWarps) {
    // ---- producer (one thread) ----------------------------------------------
    // The per-item work is a short serial chain on one thread, so positions
    // advance incrementally (no divisions on the issue path).
    if (lane != 0) return;
    const uint32_t box_tx = static_cast<uint32_t>(p.G * p.R * p.W);
    auto issue_w = [&](uint8_t* st, uint64_t* bar, int64_t row0, int ch, uint64_t choff) {
      const uint64_t cb = ch == p.nchunk - 1 ? cb_last : static_cast<uint64_t>(p.chunk_bytes);
      uint32_t tx = xbytes;
      const bool boxes = row0 < p.n_full;
      if (boxes) tx += box_tx;
      // rows past the last whole tensor row (only in the last row block of
      // the matrix): 1-D copies, the <16-byte end of the matrix by hand
      // before the arrive (whose release publishes it)
      const int64_t qa = row0 > p.n_full ? row0 : p.n_full;
      const int64_t qb = row0 + RM < r1 ? row0 + RM : r1;
      for (int64_t q = qa; q < qb; ++q) {
        const uint64_t gs = static_cast<uint64_t>(q) * p.row_bytes + choff, ge = gs + cb;
        const uint64_t a0 = gs & ~uint64_t(15);
        uint64_t a1 = (ge + 15) & ~uint64_t(15);
        if (a1 > wtot) {
          a1 = wtot & ~uint64_t(15);
          uint8_t* dst = st + p.tail_off + (q - p.n_full) * p.WT;
          for (uint64_t b = a1; b < ge; ++b) dst[b - a0] = p.w[b];
        }
        tx += static_cast<uint32_t>(a1 - a0);
      }
      mbar_arrive_expect_tx(bar, tx);
      if (boxes) {
        const int ty = static_cast<int>(row0 >> p.logG);
        uint64_t xb = choff;
        for (int j = 0; j < p.G; ++j, xb += p.row_bytes)
          tma_load_2d(st + j * p.JS, &tmap, static_cast<int>((xb & ~uint64_t(15)) >> 3), ty, bar);
      }
      for (int64_t q = qa; q < qb; ++q) {
        const uint64_t gs = static_cast<uint64_t>(q) * p.row_bytes + choff;
        const uint64_t a0 = gs & ~uint64_t(15);
        uint64_t a1 = (gs + cb + 15) & ~uint64_t(15);
        if (a1 > wtot) a1 = wtot & ~uint64_t(15);
        if (a1 > a0) bulk_g2s(st + p.tail_off + (q - p.n_full) * p.WT, p.w + a0, static_cast<uint32_t>(a1 - a0), bar);
      }
    };
    // weights of the first stages before waiting for the kernel that writes
    // the activation records (programmatic dependent launch)
    const int first = items < p.nstage ? items : p.nstage;
    int64_t row0 = r0;
    int ch = 0;
    uint64_t choff = 0;
    auto advance = [&]() {
      choff += p.chunk_bytes;
      if (++ch == p.nchunk) {
        ch = 0;
        choff = 0;
        row0 += RM;
      }
    };
    uint8_t* st = stages;
    for (int i = 0; i < first; ++i, st += p.stage_stride) {
      issue_w(st, &full[i], row0, ch, choff);
      advance();
    }
    griddep_wait();
    griddep_launch_dependents();
    {
      int cx = 0;
      st = stages;
      for (int i = 0; i < first; ++i, st += p.stage_stride) {
        bulk_g2s(st + p.x_off, p.xrec + static_cast<size_t>(cx) * xbytes, xbytes, &full[i]);
        if (++cx == p.nchunk) cx = 0;
      }
    }
    int s = 0;
    uint32_t use = 0;  // parity of the stage's previous use
    st = stages;
    int issued = first;
    for (int i = first; i < items; ++i) {
      if (!wait_phase(&empty[s], use, abort)) {
        atomicOr(p.status, kStatusEmptyWaitTimeout);
        break;
      }
      fence_proxy_async_smem();
      issue_w(st, &full[s], row0, ch, choff);
      bulk_g2s(st + p.x_off, p.xrec + static_cast<size_t>(ch) * xbytes, xbytes, &full[s]);
      advance();
      ++issued;
      st += p.stage_stride;
      if (++s == p.nstage) {
        s = 0;
        st = stages;
        use ^= 1u;
      }
    }
    const int lo = issued > p.nstage ? issued - p.nstage : 0;
    for (int i = lo; i < issued; ++i) {
      int zero = 0;
      if (!wait_phase(&full[i % p.nstage], static_cast<uint32_t>(i / p.nstage) & 1u, &zero)) {
        atomicOr(p.status, kStatusDrainTimeout);
      }
    }
    return;
  }

  // ---- consumer warps -----------------------------------------------------------
  griddep_wait();
  float acc[MT][2][NG];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int ng = 0; ng < NG; ++ng) acc[mt][h][ng] = 0.f;
  TabT* tab = reinterpret_cast<TabT*>(tab_all + warp * TABW);  // [SPW][RM]
  const int lh = M::xhalf(warp);
  // this warp's steps inside a full chunk and inside the last chunk
  int nvj_full = 0, nvj_last = 0;
#pragma unroll
  for (int j = 0; j < SPW; ++j) {
    nvj_full += M::elem(warp, j) < kMmaKC ? 1 : 0;
    nvj_last += M::elem(warp, j) < ce_last ? 1 : 0;
  }
  int s = 0;
  uint32_t ph = 0;
  int ch = 0;
  int64_t row0 = r0;
  uint64_t choff = 0;
  // Rows of the current row block this thread touches, fixed for the block:
  // decode rows L = 16 mt + 8 h + g and scale rows L = lane, lane + 32, as
  // stage-relative slot offsets plus the rows' own 16-byte phase
  // (q * row_bytes) % 16 (zero for Q4_K/Q5_K, whose blocks are 16-byte
  // multiples); a chunk adds its phase choff % 16.
  constexpr bool kPhase = F::TS % 16 != 0;
  int doff[MT][2], dmis[MT][2];
  int soff[2], smis[2];
  bool sval[2];
  auto setup_block = [&]() {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int L = 16 * mt + 8 * h + g;
        const int64_t q = slot_row(p, row0, L);
        doff[mt][h] = slot_offset(p, q, L);
        dmis[mt][h] = kPhase ? static_cast<int>((static_cast<uint64_t>(q) * p.row_bytes) & 15u) : 0;
      }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int L = lane + 32 * u;
      const int64_t q = slot_row(p, row0, L);
      sval[u] = L < RM && q < r1;
      soff[u] = slot_offset(p, q, L);
      smis[u] = kPhase ? static_cast<int>((static_cast<uint64_t>(q) * p.row_bytes) & 15u) : 0;
    }
  };
  setup_block();

  for (int i = 0; i < items; ++i) {
    const bool ok = __all_sync(0xffffffffu, wait_phase(&full[s], ph, abort));
    if (ok) {
      const int nvj = ch == p.nchunk - 1 ? nvj_last : nvj_full;
      const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_stride;
      const uint8_t* xs = st + p.x_off;
      const int chmis = static_cast<int>(choff & 15u);
      if (nvj > 0) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (sval[u]) {
            float ds[SPW], dm[SPW];
            M::scales(st + soff[u] + (kPhase ? ((smis[u] + chmis) & 15) : 0), warp, ds, dm);
#pragma unroll
            for (int j = 0; j < SPW; ++j) {
              if constexpr (M::HAS_MIN) {
                tab[j * RM + lane + 32 * u] = make_float2(ds[j], dm[j]);
              } else {
                tab[j * RM + lane + 32 * u] = ds[j];
              }
            }
          }
        }
        __syncwarp();
        // Activation fragments of step j, column group ng: B words, the group
        // scale sx, sx*sum(xq) (K-quants' min term) and the accumulator seeds
        // (Q6_K: seeds carry -32*sum of each plane, so the MMA sums
        // (q - 32) * x directly).  Loaded once for all row tiles when they
        // fit in registers (HOIST), else per row tile.
        struct BFrag {
          uint32_t b0, b1;
          float sx, sxx;
          int ch, cl;
        };
        auto load_b = [&](int j, int ng) {
          BFrag f;
          const int grp = M::xgroup(warp, j);
          const uint8_t* pb = xs + (4 * ng + (g >> 1)) * kMmaColBytes + (g & 1) * kMmaPlane + grp * 32 + 8 * t;
          const uint8_t* pm = xs + (4 * ng + t) * kMmaColBytes + 2 * kMmaPlane + grp * kMmaMeta;
          if constexpr (M::KSTEP == 32) {
            const uint2 bb = *reinterpret_cast<const uint2*>(pb);
            f.b0 = bb.x;
            f.b1 = bb.y;
            const float2 m2 = *reinterpret_cast<const float2*>(pm);
            f.sx = m2.x;
            f.sxx = m2.y;
            f.ch = kMagicBits;
            f.cl = kMagicBits;
          } else {
            f.b0 = *reinterpret_cast<const uint32_t*>(pb + 4 * lh);
            f.b1 = 0u;
            f.sx = *reinterpret_cast<const float*>(pm);
            f.sxx = 0.f;
            const int2 k2 = *reinterpret_cast<const int2*>(pm + 8 + 8 * lh);
            f.ch = kMagicBits + k2.x;
            f.cl = kMagicBits + k2.y;
          }
          return f;
        };
        constexpr bool HOIST = SPW * NG <= 8;
        BFrag bh[HOIST ? SPW : 1][HOIST ? NG : 1];
        if constexpr (HOIST) {
#pragma unroll
          for (int j = 0; j < SPW; ++j)
#pragma unroll
            for (int ng = 0; ng < NG; ++ng) bh[j][ng] = load_b(j, ng);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int la = mt * 16 + g, lb = la + 8;
          const uint8_t* pa = st + doff[mt][0] + (kPhase ? ((dmis[mt][0] + chmis) & 15) : 0);
          const uint8_t* pc = st + doff[mt][1] + (kPhase ? ((dmis[mt][1] + chmis) & 15) : 0);
          uint32_t lo0[SPW], hi0[SPW], lo1[SPW], hi1[SPW];
          M::decode(pa, warp, t, lo0, hi0);
          M::decode(pc, warp, t, lo1, hi1);
#pragma unroll
          for (int j = 0; j < SPW; ++j) {
            if (j >= nvj) break;
            float ds0, ds1, dm0 = 0.f, dm1 = 0.f;
            if constexpr (M::HAS_MIN) {
              const float2 e0 = tab[j * RM + la], e1 = tab[j * RM + lb];
              ds0 = e0.x;
              dm0 = e0.y;
              ds1 = e1.x;
              dm1 = e1.y;
            } else {
              ds0 = tab[j * RM + la];
              ds1 = tab[j * RM + lb];
            }
#pragma unroll
            for (int ng = 0; ng < NG; ++ng) {
              const BFrag f = HOIST ? bh[HOIST ? j : 0][HOIST ? ng : 0] : load_b(j, ng);
              int c[4] = {f.ch, f.cl, f.ch, f.cl};
              if constexpr (M::KSTEP == 32) {
                mma_k32<M::AU8>(c, lo0[j], lo1[j], hi0[j], hi1[j], f.b0, f.b1);
              } else {
                mma_k16(c, lo0[j], lo1[j], f.b0);
              }
              const float t0 = fmaf(256.0f, __int_as_float(c[0]) - kMagicF, __int_as_float(c[1]) - kMagicF);
              const float t1 = fmaf(256.0f, __int_as_float(c[2]) - kMagicF, __int_as_float(c[3]) - kMagicF);
              if constexpr (!M::HAS_MIN) {
                acc[mt][0][ng] = fmaf(f.sx * ds0, t0, acc[mt][0][ng]);
                acc[mt][1][ng] = fmaf(f.sx * ds1, t1, acc[mt][1][ng]);
              } else {
                acc[mt][0][ng] = fmaf(f.sx * ds0, t0, fmaf(-dm0, f.sxx, acc[mt][0][ng]));
                acc[mt][1][ng] = fmaf(f.sx * ds1, t1, fmaf(-dm1, f.sxx, acc[mt][1][ng]));
              }
            }
          }
        }
      }
    } else if (lane == 0) {
      atomicOr(p.status, kStatusFullWaitTimeout);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const bool block_done = ch == p.nchunk - 1;
    if (++s == p.nstage) {
      s = 0;
      ph ^= 1u;
    }
    choff += p.chunk_bytes;
    if (++ch == p.nchunk) {
      ch = 0;
      choff = 0;
    }
    if (block_done) {
      // row block done: reduce the warps' partial sums and write y
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int ng = 0; ng < NG; ++ng) {
            red[(warp * RM + mt * 16 + g + 8 * h) * NC + 4 * ng + t] = acc[mt][h][ng];
            acc[mt][h][ng] = 0.f;
          }
      named_barrier_sync(1, kMmaWarps * 32);
      for (int idx = threadIdx.x; idx < RM * p.batch; idx += kMmaWarps * 32) {
        const int L = idx % RM, c = idx / RM;
        const int64_t q = slot_row(p, row0, L);
        if (q >= r1) continue;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kMmaWarps; ++w) v += red[(w * RM + L) * NC + c];
        if (!*abort) p.y[static_cast<int64_t>(c) * p.n + q] = v;
      }
      named_barrier_sync(1, kMmaWarps * 32);  // red is rewritten by the next row block
      row0 += RM;
      setup_block();
    }
  }
}

}  // namespace frc
