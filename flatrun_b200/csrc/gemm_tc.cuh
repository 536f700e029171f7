// Batched prefill (more than 16 activation columns) on the 5th-generation
// tensor cores: y (seq, n) = x (seq, k) . W^T with W in raw GGUF blocks.
//
// One CTA per output tile of kTcM = 128 weight rows x kTcN = 512 tokens,
// accumulated in TMEM as a 128 x 512 fp32 accumulator (all 512 columns), so
// every weight of a 512-token prefill is dequantised once.  The k dimension
// advances in slices of kTcK = 32 elements:
//   * warp 0 streams the raw weight bytes, TcRaw<Q>::K elements of every row
//     per raw chunk, as 2-D tensor boxes (the same G-row tensor view as the
//     batched GEMV) into a 2-stage ring;
//   * warp 1 streams the fp16 activation slice (up to 512 tokens x 32 k as
//     two 256-row boxes, 64-byte swizzle) into a 3-stage ring;
//   * warps 3..10 dequantise each slice of the raw rows to fp16 (two threads
//     per row), written in the 64-byte-swizzled K-major layout the MMA reads
//     (4-stage ring), then run the epilogue;
//   * one thread of warp 2 (which also owns the TMEM allocation) issues
//     tcgen05.mma kind::f16 (M = 128, N = 256, K = 16: up to four per
//     slice, one per token half and k16 step) and releases the stages with
//     tcgen05.commit.
// Weights are rounded once to fp16 after the fp32 scale arithmetic and x is
// rounded to fp16 by a pre-pass; products accumulate in fp32.  Every wait is
// bounded; TMEM is freed on every path.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "gemv_mma.cuh"

namespace frc {

constexpr int kTcM = 128, kTcN = 512, kTcNH = 256, kTcK = 32;  // tile; kTcNH tokens per MMA
constexpr int kTcWorkers = 8;              // dequant + epilogue warps (3 .. 10)
constexpr int kTcThreads = (3 + kTcWorkers) * 32;
constexpr int kTcAStages = 4, kTcBStages = 3, kTcRawStages = 2;
constexpr int kTcATile = kTcM * kTcK * 2;    // 8 KB
constexpr int kTcBHalf = kTcNH * kTcK * 2;   // 16 KB: one 256-token box
constexpr int kTcBTile = 2 * kTcBHalf;       // 32 KB

template <int Q> struct TcRaw;  // elements of a row per raw chunk
template <> struct TcRaw<kQ4_K> { static constexpr int K = 256; };
template <> struct TcRaw<kQ5_K> { static constexpr int K = 256; };
template <> struct TcRaw<kQ6_K> { static constexpr int K = 256; };
template <> struct TcRaw<kQ8_0> { static constexpr int K = 128; };
template <> struct TcRaw<kQ1_0> { static constexpr int K = 256; };

struct TcParams {
  float* y;           // (seq, n)
  int64_t n;
  int k;
  int seq;
  int row_bytes;
  int chunk_bytes;    // raw bytes of a full raw chunk of one row
  int nchunk;         // raw chunks per row
  int G, W, R, logG, logR, JS;  // raw tile geometry (as in the batched GEMV)
  int raw_stride;     // bytes of one raw stage (G * JS rounded)
  float* ws;          // split-k partials (gridDim.z, seq, n) when gridDim.z > 1
  uint32_t* status;
};

// ---- tcgen05 / UMMA helpers --------------------------------------------------
// Shared-memory matrix descriptor of a K-major tile with the 64-byte swizzle
// (8-row atoms of 512 bytes): start address, leading offset 16 B (unused by
// swizzled K-major), stride 512 B between 8-row groups, descriptor version 1.
FRC_DEVICE_INLINE uint64_t umma_desc_sw64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;            // leading byte offset (16 B units)
  d |= static_cast<uint64_t>(512u >> 4) << 32;     // stride byte offset
  d |= static_cast<uint64_t>(1u) << 46;            // version
  d |= static_cast<uint64_t>(4u) << 61;            // layout: 64-byte swizzle
  return d;
}

// Instruction descriptor: D f32, A/B f16, both K-major, M = 128, N = 256.
constexpr uint32_t kTcIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(kTcNH >> 3) << 17) |
                              (static_cast<uint32_t>(kTcM >> 4) << 24);

FRC_DEVICE_INLINE void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

FRC_DEVICE_INLINE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

FRC_DEVICE_INLINE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FRC_DEVICE_INLINE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

FRC_DEVICE_INLINE void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- dequantisation of half a slice of a row --------------------------------
// Elements e0 + 16 hf .. e0 + 16 hf + 15 (e0 a multiple of 32, relative to the
// raw chunk) of a row whose raw chunk starts at `row`, as 8 packed fp16 pairs
// of w = scale * q - offset (fp32 arithmetic, one rounding to fp16).
FRC_DEVICE_INLINE uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Byte b of word t as the float 2^23 + byte (one permute).
template <int B>
FRC_DEVICE_INLINE float byte_f(uint32_t t) {
  return __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7650u + B));
}

// 16 unsigned byte values (4 words) -> fp16 pairs of s * (v - bias) - off,
// with v read as 2^23 + v and the 2^23 folded into the bias.
FRC_DEVICE_INLINE void bytes_to_h2(const uint32_t (&v)[4], float s, float bias, float off, uint32_t (&h)[8]) {
  const float b = 8388608.0f + bias;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[2 * i] = pack_h2(fmaf(s, byte_f<0>(v[i]) - b, -off), fmaf(s, byte_f<1>(v[i]) - b, -off));
    h[2 * i + 1] = pack_h2(fmaf(s, byte_f<2>(v[i]) - b, -off), fmaf(s, byte_f<3>(v[i]) - b, -off));
  }
}

FRC_DEVICE_INLINE void words4(const uint8_t* p, uint32_t (&w)[4]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  w[0] = v.x;
  w[1] = v.y;
  w[2] = v.z;
  w[3] = v.w;
}

template <int Q> struct TcDeq;

template <> struct TcDeq<kQ4_K> {
  // one sub-block: low (even) or high (odd) nibbles of 32 qs bytes
  static FRC_DEVICE_INLINE void half(const uint8_t* row, int e0, int hf, uint32_t (&h)[8]) {
    const int sb = e0 >> 5;
    const uint4 hdr = *reinterpret_cast<const uint4*>(row);
    float sc, m;
    scale_min_k4_words(sb, hdr.y, hdr.z, hdr.w, sc, m);
    const float ds = half_bits_to_float(hdr.x) * sc, dm = half_bits_to_float(hdr.x >> 16) * m;
    uint32_t w[4];
    words4(row + 16 + 32 * (sb >> 1) + 16 * hf, w);
    const int sh = 4 * (sb & 1);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = (w[i] >> sh) & 0x0F0F0F0Fu;
    bytes_to_h2(w, ds, 0.f, dm, h);
  }
};

template <> struct TcDeq<kQ5_K> {
  static FRC_DEVICE_INLINE void half(const uint8_t* row, int e0, int hf, uint32_t (&h)[8]) {
    const int sb = e0 >> 5;
    const uint4 hdr = *reinterpret_cast<const uint4*>(row);
    float sc, m;
    scale_min_k4_words(sb, hdr.y, hdr.z, hdr.w, sc, m);
    const float ds = half_bits_to_float(hdr.x) * sc, dm = half_bits_to_float(hdr.x >> 16) * m;
    uint32_t w[4], hb[4];
    words4(row + 48 + 32 * (sb >> 1) + 16 * hf, w);
    words4(row + 16 + 16 * hf, hb);
    const int sh = 4 * (sb & 1);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = ((w[i] >> sh) & 0x0F0F0F0Fu) | (((hb[i] >> sb) & 0x01010101u) << 4);
    bytes_to_h2(w, ds, 0.f, dm, h);
  }
};

template <> struct TcDeq<kQ6_K> {
  // quarter (hh, r) of a block; each 16-element half has its own scale
  static FRC_DEVICE_INLINE void half(const uint8_t* row, int e0, int hf, uint32_t (&h)[8]) {
    const int hh = e0 >> 7, r = (e0 & 127) >> 5;
    const float d = half_bits_to_float(ld_u16(row + 208));
    const float ds = d * static_cast<float>(static_cast<int8_t>(row[192 + 8 * hh + 2 * r + hf]));
    uint32_t ql[4], qh[4];
    lds_words_a2<4>(row + 64 * hh + 32 * (r & 1) + 16 * hf, ql);
    lds_words_a2<4>(row + 128 + 32 * hh + 16 * hf, qh);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      ql[i] = ((ql[i] >> (r >= 2 ? 4 : 0)) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * r)) & 0x03030303u) << 4);
    bytes_to_h2(ql, ds, 32.f, 0.f, h);
  }
};

template <> struct TcDeq<kQ8_0> {
  // one block: int8 values read as unsigned after flipping the sign bit
  static FRC_DEVICE_INLINE void half(const uint8_t* row, int e0, int hf, uint32_t (&h)[8]) {
    const uint8_t* blk = row + 34 * (e0 >> 5);
    const float d = half_bits_to_float(ld_u16(blk));
    uint32_t q[4];
    lds_words_a2<4>(blk + 2 + 16 * hf, q);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] ^= 0x80808080u;
    bytes_to_h2(q, d, 128.f, 0.f, h);
  }
};

template <> struct TcDeq<kQ1_0> {
  static FRC_DEVICE_INLINE void half(const uint8_t* row, int e0, int hf, uint32_t (&h)[8]) {
    const uint8_t* blk = row + 18 * (e0 >> 7);
    const float d = half_bits_to_float(ld_u16(blk));
    const uint32_t bits = ld_u16(blk + 2 + ((e0 & 127) >> 3) + 2 * hf);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      h[i] = pack_h2((bits >> (2 * i)) & 1u ? d : -d, (bits >> (2 * i + 1)) & 1u ? d : -d);
  }
};

// Shared memory: barriers and the TMEM address (1 KB), then the A, B and raw
// rings, every stage 1024-byte aligned.
struct TcSmem {
  uint64_t raw_full[kTcRawStages], raw_empty[kTcRawStages];
  uint64_t b_full[kTcBStages], b_empty[kTcBStages];
  uint64_t a_full[kTcAStages], a_empty[kTcAStages];
  uint64_t acc_full, drain;
  uint32_t tmem_base;
  int abort;
};
constexpr int kTcHeader = 1024;
static_assert(sizeof(TcSmem) <= kTcHeader, "header");

__host__ __device__ constexpr int tc_smem_bytes(int raw_stride) {
  return kTcHeader + kTcAStages * kTcATile + kTcBStages * kTcBTile + kTcRawStages * raw_stride;
}

template <int Q>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, TcParams p) {
  constexpr int RAWK = TcRaw<Q>::K;
  constexpr int SPC = RAWK / kTcK;  // slices per raw chunk
  extern __shared__ __align__(1024) uint8_t tc_smem[];
  uint8_t* smem = tc_smem;
  TcSmem* sh = reinterpret_cast<TcSmem*>(smem);
  uint8_t* a_ring = smem + kTcHeader;
  uint8_t* b_ring = a_ring + kTcAStages * kTcATile;
  uint8_t* raw_ring = b_ring + kTcBStages * kTcBTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (smem_u32(smem) & 1023u) {  // swizzled tiles need 1024-byte aligned stages
    if (threadIdx.x == 0) atomicOr(p.status, kStatusSmemMisaligned);
    return;
  }

  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kTcM;
  const int tok0 = blockIdx.y * kTcN;
  const int nslice = p.k / kTcK;
  // split-k: this CTA's raw chunks [c_begin, c_begin + ncl) and slices
  // [s_begin, s_begin + nsl); positions inside the rings count from there
  const int c_begin = static_cast<int>(static_cast<int64_t>(blockIdx.z) * p.nchunk / gridDim.z);
  const int ncl = static_cast<int>(static_cast<int64_t>(blockIdx.z + 1) * p.nchunk / gridDim.z) - c_begin;
  const int s_begin = c_begin * SPC;
  const int nsl = min((c_begin + ncl) * SPC, nslice) - s_begin;
  const int nhalf = p.seq - tok0 > kTcNH ? 2 : 1;  // 256-token halves holding tokens

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcRawStages; ++s) {
      mbar_init(&sh->raw_full[s], 1);
      mbar_init(&sh->raw_empty[s], kTcWorkers);
    }
    for (int s = 0; s < kTcBStages; ++s) {
      mbar_init(&sh->b_full[s], 1);
      mbar_init(&sh->b_empty[s], 1);
    }
    for (int s = 0; s < kTcAStages; ++s) {
      mbar_init(&sh->a_full[s], kTcWorkers);
      mbar_init(&sh->a_empty[s], 1);
    }
    mbar_init(&sh->acc_full, 1);
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {  // the whole TMEM: two 128 x 256 fp32 accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&sh->tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  volatile int* abort = &sh->abort;

  if (warp == 0) {
    // ---- raw weights --------------------------------------------------------
    if (lane == 0) {
      const uint32_t tx = static_cast<uint32_t>(p.G * p.R * p.W);
      const int ty = static_cast<int>(row0 >> p.logG);
      uint64_t choff = static_cast<uint64_t>(c_begin) * p.chunk_bytes;
      int issued = 0;
      for (int c = 0; c < ncl; ++c, choff += p.chunk_bytes) {
        const int s = c % kTcRawStages;
        if (c >= kTcRawStages &&
            !wait_phase(&sh->raw_empty[s], (static_cast<uint32_t>(c / kTcRawStages) & 1u) ^ 1u, abort)) {
          atomicOr(p.status, kStatusEmptyWaitTimeout);
          break;
        }
        uint8_t* st = raw_ring + static_cast<size_t>(s) * p.raw_stride;
        mbar_arrive_expect_tx(&sh->raw_full[s], tx);
        uint64_t xb = choff;
        for (int j = 0; j < p.G; ++j, xb += p.row_bytes)
          tma_load_2d(st + j * p.JS, &wmap, static_cast<int>((xb & ~uint64_t(15)) >> 3), ty, &sh->raw_full[s]);
        ++issued;
      }
      // no copy may still be landing when the CTA exits
      for (int c = issued > kTcRawStages ? issued - kTcRawStages : 0; c < issued; ++c) {
        int zero = 0;
        if (!wait_phase(&sh->raw_full[c % kTcRawStages], static_cast<uint32_t>(c / kTcRawStages) & 1u, &zero))
          atomicOr(p.status, kStatusDrainTimeout);
      }
    }
  } else if (warp == 1) {
    // ---- fp16 activations -----------------------------------------------------
    if (lane == 0) {
      int issued = 0;
      for (int s = 0; s < nsl; ++s) {
        const int b = s % kTcBStages;
        if (s >= kTcBStages &&
            !wait_phase(&sh->b_empty[b], (static_cast<uint32_t>(s / kTcBStages) & 1u) ^ 1u, abort)) {
          atomicOr(p.status, kStatusEmptyWaitTimeout);
          break;
        }
        mbar_arrive_expect_tx(&sh->b_full[b], nhalf * kTcBHalf);
        for (int nh = 0; nh < nhalf; ++nh)
          tma_load_2d(b_ring + b * kTcBTile + nh * kTcBHalf, &xmap, (s_begin + s) * kTcK, tok0 + nh * kTcNH,
                      &sh->b_full[b]);
        ++issued;
      }
      for (int s = issued > kTcBStages ? issued - kTcBStages : 0; s < issued; ++s) {
        int zero = 0;
        if (!wait_phase(&sh->b_full[s % kTcBStages], static_cast<uint32_t>(s / kTcBStages) & 1u, &zero))
          atomicOr(p.status, kStatusDrainTimeout);
      }
    }
  } else if (warp == 2) {
    // ---- MMA issue (one thread) ------------------------------------------------
    if (lane == 0) {
      int s = 0;
      for (; s < nsl; ++s) {
        const int a = s % kTcAStages, b = s % kTcBStages;
        if (!wait_phase(&sh->a_full[a], static_cast<uint32_t>(s / kTcAStages) & 1u, abort) ||
            !wait_phase(&sh->b_full[b], static_cast<uint32_t>(s / kTcBStages) & 1u, abort)) {
          atomicOr(p.status, kStatusFullWaitTimeout);
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(a_ring + a * kTcATile), b_addr = smem_u32(b_ring + b * kTcBTile);
        for (int nh = 0; nh < nhalf; ++nh)
#pragma unroll
          for (int kk = 0; kk < kTcK / 16; ++kk)
            umma_f16(tmem + nh * kTcNH, umma_desc_sw64(a_addr + kk * 32), umma_desc_sw64(b_addr + nh * kTcBHalf + kk * 32),
                     (s > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&sh->a_empty[a]);
        umma_commit(&sh->b_empty[b]);
      }
      // accumulators complete (or, after an abort, every issued MMA retired);
      // this thread also waits, so no MMA is in flight at the teardown
      uint64_t* done = s == nsl ? &sh->acc_full : &sh->drain;
      umma_commit(done);
      int zero = 0;
      if (!wait_phase(done, 0u, &zero)) atomicOr(p.status, kStatusDrainTimeout);
    }
  } else {
    // ---- dequantisation into the swizzled fp16 A stages ----------------------------
    const int L = (threadIdx.x - 3 * 32) >> 1;  // this thread's tile row, 0 .. 127
    const int hf = threadIdx.x & 1;               // and its half of each slice
    const int64_t q = row0 + (static_cast<int64_t>(L & (p.R - 1)) << p.logG) + (L >> p.logR);
    const int slot = (L >> p.logR) * p.JS + (L & (p.R - 1)) * p.W;
    const uint32_t qmis = static_cast<uint32_t>((static_cast<uint64_t>(q) * p.row_bytes) & 15u);
    const int swz = (L >> 1) & 3;
    bool ok = true;
    for (int s = 0; s < nsl && ok; ++s) {
      const int c = s / SPC, a = s % kTcAStages, rs = c % kTcRawStages;
      if (s % SPC == 0)
        ok = __all_sync(0xffffffffu, wait_phase(&sh->raw_full[rs], static_cast<uint32_t>(c / kTcRawStages) & 1u, abort));
      if (ok && s >= kTcAStages)
        ok = __all_sync(0xffffffffu,
                        wait_phase(&sh->a_empty[a], (static_cast<uint32_t>(s / kTcAStages) & 1u) ^ 1u, abort));
      if (!ok) {
        if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
        break;
      }
      const uint8_t* raw = raw_ring + static_cast<size_t>(rs) * p.raw_stride;
      const uint32_t chmis = static_cast<uint32_t>((static_cast<uint64_t>(c_begin + c) * p.chunk_bytes) & 15u);
      uint32_t h[8];
      TcDeq<Q>::half(raw + slot + ((qmis + chmis) & 15u), (s % SPC) * kTcK, hf, h);
      // 64-byte swizzle: 16-byte chunk index ^= (row / 2) % 4 within 512-byte atoms
      uint8_t* line = a_ring + a * kTcATile + L * 64;
#pragma unroll
      for (int j = 0; j < 2; ++j)
        *reinterpret_cast<uint4*>(line + (((2 * hf + j) ^ swz) << 4)) =
            make_uint4(h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sh->a_full[a]);
        if (s % SPC == SPC - 1 || s == nsl - 1) mbar_arrive(&sh->raw_empty[rs]);
      }
    }
    // ---- epilogue: TMEM -> y -------------------------------------------------------
    ok = ok && __all_sync(0xffffffffu, wait_phase(&sh->acc_full, 0u, abort));
    if (ok) {
      tc_fence_after();
      const int quad = warp & 3;           // TMEM lanes 32*quad .. +31
      const int nh = (warp - 3) >> 2;      // tokens [256*nh, 256*nh + 256)
      const int L = quad * 32 + lane;
      const int64_t q = row0 + (static_cast<int64_t>(L & (p.R - 1)) << p.logG) + (L >> p.logR);
      float* out = gridDim.z > 1 ? p.ws + static_cast<int64_t>(blockIdx.z) * p.seq * p.n : p.y;
      if (nh < nhalf) {
#pragma unroll 1
        for (int cb = 0; cb < kTcNH; cb += 16) {
          float v[16];
          tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + nh * kTcNH + cb, v);
          if (q < p.n && !*abort) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int t = tok0 + nh * kTcNH + cb + i;
              if (t < p.seq) out[static_cast<int64_t>(t) * p.n + q] = v[i];
            }
          }
        }
      }
    } else if (lane == 0) {
      atomicOr(p.status, kStatusFullWaitTimeout);
    }
  }
  // ---- teardown: every warp here, no MMA or TMEM load in flight -----------------
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// y = sum of the split-k partials, in split order (deterministic).
static __global__ void __launch_bounds__(256) tc_reduce(const float* __restrict__ ws, int splits, int64_t count,
                                                      float* __restrict__ y) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    float v = ws[i];
    for (int z = 1; z < splits; ++z) v += ws[z * count + i];
    y[i] = v;
  }
}

// fp32 activations -> fp16 (seq, k), 8 elements per thread.
static __global__ void __launch_bounds__(256) tc_convert_x(const float* __restrict__ x, int64_t count,
                                                         __half* __restrict__ out) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i >= count) return;
  const float4 a = *reinterpret_cast<const float4*>(x + i);
  const float4 b = *reinterpret_cast<const float4*>(x + i + 4);
  *reinterpret_cast<uint4*>(out + i) =
      make_uint4(pack_h2(a.x, a.y), pack_h2(a.z, a.w), pack_h2(b.x, b.y), pack_h2(b.z, b.w));
}

}  // namespace frc
