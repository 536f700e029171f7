// Host-side launch of the per-format kernels: configuration choice, dynamic
// shared-memory opt-in and occupancy, cached per (device, kernel).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "gemv.cuh"
#include "gemv_tc1.cuh"
#include "gemm_tc.cuh"
#include "gemv_mma.cuh"

namespace frc {

struct GemvRequest {
  const uint8_t* w;
  const float* x;
  float* y;
  int64_t n;
  int k;
  int batch;  // 1..16
  uint32_t* status;
  cudaStream_t stream;
  int device;
  int sms;
  // batch-1 fused launch over several matrices sharing x (nmat > 1): rows
  // are concatenated; w, y, n then describe nothing and these arrays are used
  int nmat;
  const uint8_t* mat_w[4];
  float* mat_y[4];
  int64_t mat_n[4];
  // batch 2..16: activation records of the tensor-core kernel (at least
  // mma_scratch_bytes(k, batch) bytes, 256-byte aligned); null selects the
  // fp32 CUDA-core kernel.  Prefill (batch > 16): fp16 x and split-k
  // partials (tc_scratch_bytes(k, n, batch, tc_splits) bytes)
  uint8_t* xrec;
  int tc_splits;  // prefill k-splits (>= 1)
  // batch-1 fused all-gather (g_world > 1; see GemvParams)
  int g_world, g_rank;
  const float* g_ybase;
  float* g_peer_y[kMaxGatherRanks];
  uint32_t* g_flags[kMaxGatherRanks];
  uint32_t* g_done;
  uint32_t* g_epoch;
  int w_world;  // batch-1: wait for an earlier fused gather before reading x
  const uint32_t* w_flags;
  const uint32_t* w_epoch;
  // batch-1, fp32 activations: x read as silu(x) * x_mul; y accumulated
  const float* x_mul;
  int y_accum;
  const float* x_norm_w;  // batch-1, fp32 activations: x read as RMSNorm(x) * x_norm_w
  float x_norm_eps;
};

struct DequantRequest {
  const uint8_t* w;
  int64_t n_elems;
  float* out;
  cudaStream_t stream;
  int sms;
};

// Library options, set through frc_set_option (include/frcuda.h); read on
// every launch with relaxed atomics, never from the environment.
struct Options {
  std::atomic<int> batch1_int16{0};    // FRC_OPT_BATCH1_INT16
  std::atomic<int> batched_fp32{0};    // FRC_OPT_BATCHED_FP32
  std::atomic<int> prefill_tc{1};      // FRC_OPT_PREFILL_TC
  std::atomic<int> prefill_splits{0};  // FRC_OPT_PREFILL_SPLITS
  std::atomic<int> inject_oom{0};      // FRC_OPT_INJECT_OOM
  std::atomic<int> batch1_tc{1};       // FRC_OPT_BATCH1_TC (0, 1, 2)
};
inline Options& options() {
  static Options o;
  return o;
}
inline int opt(const std::atomic<int>& v) { return v.load(std::memory_order_relaxed); }

// Launch-configuration overrides for tuning sweeps.  They are read from the
// environment once, at the first launch, and only when FRC_TUNE=1; otherwise
// every kernel runs its measured default configuration.  -1 = not set.
struct Tuning {
  int upt = -1, rps = -1, tile_bytes = -1, nwarps = -1, nstage = -1, smem_bytes = -1, rt = -1, stage_bytes = -1,
      ctas_per_sm = -1, mma_grid = -1, mma_mt = -1, pre_stages = -1, pdl = -1, tc_mt = -1, tc_builders = -1,
      tc_stages = -1, tc_part_chunks = -1, tc_split = -1;
};
inline const Tuning& tuning() {
  static const Tuning t = [] {
    Tuning v;
    const char* on = std::getenv("FRC_TUNE");
    if (!on || std::strcmp(on, "1") != 0) return v;
    auto get = [](const char* name) {
      const char* s = std::getenv(name);
      return (s && *s) ? std::atoi(s) : -1;
    };
    v.upt = get("FRC_UPT");
    v.rps = get("FRC_RPS");
    v.tile_bytes = get("FRC_TILE_BYTES");
    v.nwarps = get("FRC_NWARPS");
    v.nstage = get("FRC_NSTAGE");
    v.smem_bytes = get("FRC_SMEM_BYTES");
    v.rt = get("FRC_RT");
    v.stage_bytes = get("FRC_STAGE_BYTES");
    v.ctas_per_sm = get("FRC_CTAS_PER_SM");
    v.mma_grid = get("FRC_MMA_GRID");
    v.mma_mt = get("FRC_MMA_MT");
    v.pre_stages = get("FRC_PRE_STAGES");
    v.pdl = get("FRC_PDL");
    v.tc_mt = get("FRC_TC_MT");
    v.tc_builders = get("FRC_TC_BUILDERS");
    v.tc_stages = get("FRC_TC_STAGES");
    v.tc_part_chunks = get("FRC_TC_PC");
    v.tc_split = get("FRC_TC_SPLIT");
    return v;
  }();
  return t;
}
// A tuning override if set, else the default.
inline int tuned(int v, int def) { return v >= 0 ? v : def; }

// Blocks of `kernel` resident per SM with `threads` threads and `smem` bytes,
// after opting the kernel into `smem` bytes of dynamic shared memory.
inline cudaError_t kernel_occupancy(const void* kernel, int device, int threads, size_t smem, int* blocks) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, int, size_t>, int> cache;
  // the opt-in is a per-(kernel, device) cap: only ever raise it, or a later
  // smaller request would invalidate a cached larger configuration
  static std::map<std::pair<const void*, int>, size_t> optin;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(kernel, device, threads, smem);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *blocks = it->second;
    return cudaSuccess;
  }
  size_t& cap = optin[std::make_pair(kernel, device)];
  if (smem > cap) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cap = smem;
  }
  cudaError_t e;
  int nb = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, threads, smem);
  if (e != cudaSuccess) return e;
  if (nb < 1) return cudaErrorInvalidConfiguration;
  cache[key] = nb;
  *blocks = nb;
  return cudaSuccess;
}

// Clusters of `cfg`'s shape (cluster size, block size, shared memory) the
// device holds at once, looked up once per kernel, device and shape.
inline cudaError_t max_active_clusters(const void* kernel, int device, const cudaLaunchConfig_t& cfg, int* clusters) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, unsigned, unsigned, size_t>, int> cache;
  unsigned csize = 1;
  for (unsigned i = 0; i < cfg.numAttrs; ++i)
    if (cfg.attrs[i].id == cudaLaunchAttributeClusterDimension) csize = cfg.attrs[i].val.clusterDim.x;
  const auto key = std::make_tuple(kernel, device, csize, cfg.blockDim.x, cfg.dynamicSmemBytes);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *clusters = it->second;
    return cudaSuccess;
  }
  int n = 0;
  const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
  if (e != cudaSuccess) return e;
  cache[key] = n;
  *clusters = n;
  return cudaSuccess;
}

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Shared-memory stage geometry for tiles of `rt` rows.
inline void stage_geometry(int row_bytes, int rt, int* stride, int* nstage) {
  *stride = round_up(rt * row_bytes + 32, 128);
  const int target = tuned(tuning().stage_bytes, 64 * 1024);
  int ns = target / *stride;
  ns = ns < 2 ? 2 : (ns > 8 ? 8 : ns);
  const int forced = tuning().nstage;
  *nstage = forced > 0 ? forced : ns;
}

template <typename K>
inline cudaError_t launch_persistent(K kernel, GemvParams p, int ncw, size_t smem, const GemvRequest& r) {
  const int threads = (ncw + 1) * 32;
  int per_sm = 0;
  cudaError_t e = kernel_occupancy(reinterpret_cast<const void*>(kernel), r.device, threads, smem, &per_sm);
  if (e != cudaSuccess) return e;
  const int cap = tuning().ctas_per_sm;
  if (cap > 0 && cap < per_sm) per_sm = cap;
  int64_t grid = static_cast<int64_t>(per_sm) * r.sms;
  if (grid > p.n) grid = p.n;
  if (grid < 1) grid = 1;
  kernel<<<static_cast<unsigned>(grid), threads, smem, r.stream>>>(p);
  return cudaGetLastError();
}

inline int rows_per_tile(int row_bytes);

template <int Q, int RT, int BMAX>
inline cudaError_t launch_xb_rt(GemvParams p, const GemvRequest& r) {
  const int ncw = p.units >= 32 * kMaxConsumerWarps ? kMaxConsumerWarps : (p.units + 31) / 32;
  stage_geometry(p.row_bytes, RT, &p.stage_stride, &p.nstage);
  const size_t smem = smem_header_bytes<RT * BMAX>() + static_cast<size_t>(p.nstage) * p.stage_stride;
  return launch_persistent(gemv_xb<Q, RT, BMAX>, p, ncw, smem, r);
}

// Rows per tile: as many as the accumulator budget (RT * BMAX <= 32) and
// the row length allow.
inline int rows_per_tile(int row_bytes) {
  int rt = 8;
  if (row_bytes > 4096) rt = 4;
  if (row_bytes > 16384) rt = 2;
  const int forced = tuning().rt;
  if (forced == 2 || forced == 4 || forced == 8) rt = forced;
  return rt;
}

template <int Q, int BMAX>
inline cudaError_t launch_xb(GemvParams p, const GemvRequest& r) {
  int rt = rows_per_tile(p.row_bytes);
  if (rt * BMAX > 32) rt = 32 / BMAX;
  if constexpr (BMAX == 4) {
    if (rt == 8) return launch_xb_rt<Q, 8, 4>(p, r);
    if (rt == 4) return launch_xb_rt<Q, 4, 4>(p, r);
    return launch_xb_rt<Q, 2, 4>(p, r);
  } else if constexpr (BMAX == 8) {
    if (rt == 4) return launch_xb_rt<Q, 4, 8>(p, r);
    return launch_xb_rt<Q, 2, 8>(p, r);
  } else {
    return launch_xb_rt<Q, 2, 16>(p, r);
  }
}

// Batch-1 kernel (gemv_b1): slots of `wps` warps each cover one row's units
// and run independent pipelines; up to 16 warps per CTA.  F32 selects the
// fp32-activation arithmetic, otherwise the 16-bit integer grid.
template <int Q, int UPT, int RPS, bool F32>
inline cudaError_t launch_b1_rps(GemvParams p, const GemvRequest& r, int slots, int nst) {
  p.stage_stride = round_up(RPS * p.row_bytes + 32, 128);
  p.nstage = nst;
  // one stage per slot before the grid dependency wait: a full ring of
  // weight copies in flight delays the activation loads behind it (measured
  // on B200: the Qwen2-7B layer step 43.8 -> 41.8 us)
  p.pre_stages = tuned(tuning().pre_stages, 1);
  const size_t smem =
      b1_smem_header<Q, RPS, F32>(slots, nst, p.wps, p.units) + static_cast<size_t>(slots) * nst * p.stage_stride;
  const int threads = slots * p.wps * 32;
  const void* fn = reinterpret_cast<const void*>(gemv_b1<Q, UPT, RPS, F32>);
  int per_sm = 0;
  cudaError_t e = kernel_occupancy(fn, r.device, threads, smem, &per_sm);
  if (e != cudaSuccess) return e;
  int64_t grid = static_cast<int64_t>(per_sm) * r.sms;
  const int64_t useful = (p.n + slots - 1) / slots;
  if (grid > useful) grid = useful;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = r.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = tuned(tuning().pdl, 1) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_b1<Q, UPT, RPS, F32>, p);
}

// Shared memory available to one block (B200: 227 KB opt-in).
constexpr int kSmemBudget = 227 * 1024;

// Bytes of weights per tile the batch-1 kernel aims for (rows per tile = the
// largest power of two <= 8 whose tile fits), swept on B200.  Integer
// kernel: ~8 KB for short K-quant rows, 12 KB (four 2940-byte rows) for the
// k = 3584 Q6_K lm_head (4.3 -> 5.1 TB/s), 18 KB (four rows) for k = 4096
// Q8_0, 4 KB (four rows) for Q1_0; long rows (k > ~14K for Q4_K) two-row
// tiles up to 32 KB.
template <int Q, bool F32>
inline int b1_tile_target(int row_bytes) {
  // the fp32-activation kernel spends more per tile (its dot is longer and
  // the per-tile reduction is the same), so it wants more rows per tile:
  // swept on B200, a Llama-3-70B layer's gate+up (4608-byte rows) runs 0.29
  // -> 0.50 of the copy peak with ~32 KB tiles, its down (16128-byte rows)
  // 2.2 -> 2.8 TB/s with ~64 KB; the Qwen2-7B shapes are insensitive
  if constexpr (F32) return row_bytes > 8192 ? 64 * 1024 : 32 * 1024;
  if (row_bytes > 8192) return 32 * 1024;
  if constexpr (Q == kQ6_K) return 12 * 1024;
  if constexpr (Q == kQ8_0) return 18 * 1024;
  if constexpr (Q == kQ1_0) return 4 * 1024;
  return 8 * 1024;
}

// Choose slots (independent pipelines of wps warps), rows per tile and stages
// so the block fits in shared memory: prefer the requested tile size and as
// many warps as the register budget allows, then shrink tiles, then warps.
template <int Q, int UPT, bool F32>
inline cudaError_t launch_b1(GemvParams p, const GemvRequest& r) {
  const int spt = 32 * UPT;
  p.wps = (p.units + spt - 1) / spt;
  constexpr int kMaxW = b1_max_warps<Q, UPT, F32>();
  const int warps = tuned(tuning().nwarps, kMaxW);
  int slots = warps / p.wps;
  if (slots < 1) slots = 1;
  if (slots * p.wps > kMaxW) slots = kMaxW / p.wps;
  if (slots < 1) return cudaErrorInvalidValue;
  const int tile_target = tuned(tuning().tile_bytes, b1_tile_target<Q, F32>(p.row_bytes));
  int rps = 1;
  while (rps < 8 && 2 * rps * p.row_bytes <= tile_target) rps *= 2;
  const int forced = tuning().rps;
  if (forced == 1 || forced == 2 || forced == 4 || forced == 8) rps = forced;
  const int budget = tuned(tuning().smem_bytes, kSmemBudget);
  const int want_nst = tuning().nstage;
  for (; slots >= 1; --slots) {
    for (int rr = rps; rr >= 1; rr /= 2) {
      const int stride = round_up(rr * p.row_bytes + 32, 128);
      int header = 0;
      switch (rr) {
        case 1: header = b1_smem_header<Q, 1, F32>(slots, 8, p.wps, p.units); break;
        case 2: header = b1_smem_header<Q, 2, F32>(slots, 8, p.wps, p.units); break;
        case 4: header = b1_smem_header<Q, 4, F32>(slots, 8, p.wps, p.units); break;
        default: header = b1_smem_header<Q, 8, F32>(slots, 8, p.wps, p.units); break;
      }
      int nst = (budget - header) / (slots * stride);
      if (nst > 8) nst = 8;
      if (want_nst > 0 && want_nst < nst) nst = want_nst;
      if (nst < 2) continue;
      switch (rr) {
        case 1: return launch_b1_rps<Q, UPT, 1, F32>(p, r, slots, nst);
        case 2: return launch_b1_rps<Q, UPT, 2, F32>(p, r, slots, nst);
        case 4: return launch_b1_rps<Q, UPT, 4, F32>(p, r, slots, nst);
        default: return launch_b1_rps<Q, UPT, 8, F32>(p, r, slots, nst);
      }
    }
  }
  return cudaErrorInvalidValue;
}

// Units per thread of the batch-1 kernel: the fewest that cover a row with
// the warps the register budget allows.  The integer kernel's choice was swept
// on B200: K-quant rows of up to 64 units use 1 unit per thread in two-warp
// slots, longer rows 2; Q8_0 rows of up to 128 units 1 (4096x4096: 6.5 -> 6.1
// us); Q1_0 2 (4096x4096: 6.0 -> 5.4 us).  fp32 units hold 4x the activation
// registers, so they take 1 unit per thread while a row fits 16 warps.
template <int Q, bool F32>
inline cudaError_t launch_b1_any(GemvParams p, const GemvRequest& r) {
  const int units = p.units;
  int upt = tuning().upt;
  if (upt <= 0) {
    if constexpr (F32) upt = units <= 32 * b1_max_warps<Q, 1, F32>() ? 1 : 2;
    else if constexpr (Q == kQ8_0) upt = units <= 128 ? 1 : 2;
    else if constexpr (Q == kQ1_0) upt = 2;
    else upt = units <= 64 ? 1 : 2;
  }
  if constexpr (!F32 && I8<Q>::E == 32) {
    if (upt == 4 && units <= 128) return launch_b1<Q, 4, F32>(p, r);
  }
  if (upt >= 2 && units <= 64 * b1_max_warps<Q, 2, F32>()) return launch_b1<Q, 2, F32>(p, r);
  if (units <= 32 * b1_max_warps<Q, 1, F32>()) return launch_b1<Q, 1, F32>(p, r);
  if (units <= 64 * b1_max_warps<Q, 2, F32>()) return launch_b1<Q, 2, F32>(p, r);
  return cudaErrorInvalidValue;
}

// Bytes of activation records the tensor-core batched kernel needs.
inline int64_t mma_scratch_bytes(int64_t k, int batch) {
  const int ng = batch <= 4 ? 1 : (batch <= 8 ? 2 : 4);
  return (k + kMmaKC - 1) / kMmaKC * 4 * ng * kMmaColBytes;
}

// Launch with programmatic dependent launch allowed (FRC_PDL=0 turns it off).
template <typename... P, typename... A>
inline cudaError_t launch_pdl(void (*kernel)(P...), unsigned grid, unsigned threads, size_t smem, cudaStream_t st,
                              A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = tuned(tuning().pdl, 1) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// cuTensorMapEncodeTiled from the driver, looked up once.
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// Tile geometry of the batched kernel for rows of `row_bytes` and full chunks
// of `chunk_bytes`: G = rows per tensor row (G * row_bytes % 16 == 0) and box
// width W (covers a chunk from its 16-byte-aligned start, and an odd multiple
// of 16 bytes so eight consecutive box rows start in distinct bank groups).
inline void mma_geometry(int row_bytes, int chunk_bytes, int* G, int* W) {
  int g = 1;
  while ((g * row_bytes) % 16 != 0) g *= 2;
  int mis = 0;
  for (int a = 0; a < 16; ++a)
    for (int c = 0; c < 16; ++c) {
      const int m = (a * row_bytes + c * chunk_bytes) & 15;
      mis = m > mis ? m : mis;
    }
  int w = round_up(chunk_bytes + mis, 16);
  if ((w / 16) % 2 == 0) w += 16;
  *G = g;
  *W = w;
}

// Tensor-core batched kernel: pre-pass over x, then persistent CTAs of one
// producer and eight consumer warps over row blocks of 16 MT rows.
template <int Q, int NG, int MT>
inline cudaError_t launch_mma_cfg(MmaParams p, const GemvRequest& r, int grid) {
  constexpr int RM = 16 * MT;
  if (RM % (8 * p.G) != 0) return cudaErrorInvalidValue;
  p.R = RM / p.G;
  p.logG = 0;
  while ((1 << p.logG) < p.G) ++p.logG;
  p.logR = 0;
  while ((1 << p.logR) < p.R) ++p.logR;
  p.JS = round_up(p.R * p.W, 128);
  p.n_full = r.n / p.G * p.G;
  p.WT = round_up(p.chunk_bytes + 32, 16);
  p.tail_off = p.G * p.JS;
  p.x_off = round_up(p.tail_off + (p.G - 1) * p.WT, 128);
  const int xbytes = 4 * NG * kMmaColBytes;
  p.stage_stride = round_up(p.x_off + xbytes, 128);
  constexpr int header = mma_header_bytes<Q, NG, MT>();
  const int budget = tuned(tuning().smem_bytes, kSmemBudget);
  int nst = (budget - header) / p.stage_stride;
  if (nst > 6) nst = 6;
  const int want = tuning().nstage;
  if (want > 0 && want < nst) nst = want;
  if (nst < 2) return cudaErrorInvalidValue;
  p.nstage = nst;
  const size_t smem = header + static_cast<size_t>(nst) * p.stage_stride;
  const int threads = (kMmaWarps + 1) * 32;
  int per_sm = 0;
  cudaError_t e = kernel_occupancy(reinterpret_cast<const void*>(gemv_mma<Q, NG, MT>), r.device, threads, smem,
                                   &per_sm);
  if (e != cudaSuccess) return e;
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  if (p.n_full > 0) {
    auto encode = tensor_map_encoder();
    if (!encode) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.G) * p.row_bytes / 8,
                                static_cast<cuuint64_t>(p.n_full / p.G)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.G) * p.row_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(p.W / 8), static_cast<cuuint32_t>(p.R)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(p.w), dims, strides,
                               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  const int64_t qthreads = static_cast<int64_t>(p.nchunk) * p.ncols * (kMmaKC / 32);
  e = launch_pdl(mma_quantise_x, static_cast<unsigned>((qthreads + 255) / 256), 256, 0, r.stream, r.x, p.k,
                 p.batch, p.ncols, p.nchunk, r.xrec);
  if (e != cudaSuccess) return e;
  return launch_pdl(gemv_mma<Q, NG, MT>, static_cast<unsigned>(grid), threads, smem, r.stream, map, p);
}

template <int Q, int NG>
inline cudaError_t launch_mma_ng(MmaParams p, const GemvRequest& r) {
  mma_geometry(p.row_bytes, p.chunk_bytes, &p.G, &p.W);
  // smallest row block whose boxes hold whole 8-row half tiles
  const int mt_min = p.G >= 8 ? 4 : (p.G == 4 ? 2 : 1);
  int64_t grid = tuned(tuning().mma_grid, r.sms);
  const int64_t useful = (p.n + 16 * mt_min - 1) / (16 * mt_min);
  if (grid > useful) grid = useful;
  if (grid < 1) grid = 1;
  const int64_t per_cta = (p.n + grid - 1) / grid;
  int mt = tuned(tuning().mma_mt, per_cta <= 16 ? 1 : (per_cta <= 32 ? 2 : 4));
  if (mt < mt_min) mt = mt_min;
  if (mt == 1) return launch_mma_cfg<Q, NG, 1>(p, r, static_cast<int>(grid));
  if (mt == 2) return launch_mma_cfg<Q, NG, 2>(p, r, static_cast<int>(grid));
  return launch_mma_cfg<Q, NG, 4>(p, r, static_cast<int>(grid));
}

template <int Q>
inline cudaError_t launch_mma(const GemvRequest& r) {
  using F = Fmt<Q>;
  MmaParams p{};
  p.w = r.w;
  p.y = r.y;
  p.n = r.n;
  p.k = r.k;
  p.batch = r.batch;
  p.row_bytes = (r.k / F::QK) * F::TS;
  p.chunk_bytes = kMmaKC / F::QK * F::TS;
  p.nchunk = (r.k + kMmaKC - 1) / kMmaKC;
  p.xrec = r.xrec;
  p.status = r.status;
  if (r.batch <= 4) {
    p.ncols = 4;
    return launch_mma_ng<Q, 1>(p, r);
  }
  if (r.batch <= 8) {
    p.ncols = 8;
    return launch_mma_ng<Q, 2>(p, r);
  }
  p.ncols = 16;
  return launch_mma_ng<Q, 4>(p, r);
}

// Raw-chunk elements of the prefill GEMM per format (TcRaw<Q>::K).
inline int tc_raw_k(int quant) { return quant == kQ8_0 ? 128 : 256; }

// k-splits of a prefill: enough CTAs to fill the SMs when the (row, token)
// tiles alone do not (at most 16, at least one raw chunk per split);
// FRC_TC_SPLIT overrides.
inline int tc_split_count(int quant, int64_t n, int64_t k, int64_t seq, int sms) {
  const int64_t tiles = ((n + kTcM - 1) / kTcM) * ((seq + kTcN - 1) / kTcN);
  const int64_t nchunk = (k + tc_raw_k(quant) - 1) / tc_raw_k(quant);
  int64_t s = opt(options().prefill_splits);
  if (s <= 0) s = tiles >= sms ? 1 : sms / tiles;
  if (s > 16) s = 16;
  if (s > nchunk) s = nchunk;
  return s < 1 ? 1 : static_cast<int>(s);
}

// Bytes of prefill scratch: fp16 x, then (split-k only) fp32 partials.
inline int64_t tc_x16_bytes(int64_t k, int64_t seq) { return (seq * k * 2 + 255) / 256 * 256; }
inline int64_t tc_scratch_bytes(int64_t k, int64_t n, int64_t seq, int splits) {
  return tc_x16_bytes(k, seq) + (splits > 1 ? static_cast<int64_t>(splits) * seq * n * 4 : 0);
}

// Tensor-core prefill (seq > 16): x -> fp16 pre-pass, then one CTA per
// 128-row x 512-token tile.  cudaErrorNotSupported when the shape does not
// fit this kernel (the caller then runs 16-column chunks).
template <int Q>
inline cudaError_t launch_gemm_tc(const GemvRequest& r) {
  using F = Fmt<Q>;
  constexpr int RAWK = TcRaw<Q>::K;
  TcParams p{};
  p.y = r.y;
  p.n = r.n;
  p.k = r.k;
  p.seq = r.batch;
  p.row_bytes = (r.k / F::QK) * F::TS;
  p.chunk_bytes = RAWK / F::QK * F::TS;
  p.nchunk = (r.k + RAWK - 1) / RAWK;
  p.status = r.status;
  const int splits = r.tc_splits < 1 ? 1 : r.tc_splits;
  p.ws = splits > 1 ? reinterpret_cast<float*>(r.xrec + tc_x16_bytes(r.k, r.batch)) : nullptr;
  mma_geometry(p.row_bytes, p.chunk_bytes, &p.G, &p.W);
  if (r.n % p.G != 0 || r.k % kTcK != 0 || !r.xrec || splits > p.nchunk) return cudaErrorNotSupported;
  p.R = kTcM / p.G;
  p.logG = 0;
  while ((1 << p.logG) < p.G) ++p.logG;
  p.logR = 0;
  while ((1 << p.logR) < p.R) ++p.logR;
  p.JS = round_up(p.R * p.W, 128);
  p.raw_stride = round_up(p.G * p.JS, 1024);
  // + 1 KB slack: the dequant's word loads may run a few bytes past the last
  // raw row; at least ~120 KB so two CTAs never share an SM (each takes all
  // of TMEM)
  int smem = tc_smem_bytes(p.raw_stride) + 1024;
  if (smem < 120 * 1024) smem = 120 * 1024;
  if (smem > kSmemBudget) return cudaErrorNotSupported;
  int per_sm = 0;
  cudaError_t e = kernel_occupancy(reinterpret_cast<const void*>(gemm_tc<Q>), r.device, kTcThreads, smem, &per_sm);
  if (e != cudaSuccess) return e;
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  CUtensorMap wmap, xmap;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.G) * p.row_bytes / 8, static_cast<cuuint64_t>(r.n / p.G)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.G) * p.row_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(p.W / 8), static_cast<cuuint32_t>(p.R)};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(r.w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(r.k), static_cast<cuuint64_t>(r.batch)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(r.k) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTcK), static_cast<cuuint32_t>(kTcNH)};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, r.xrec, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  const int64_t count = static_cast<int64_t>(r.batch) * r.k;
  tc_convert_x<<<static_cast<unsigned>((count / 8 + 255) / 256), 256, 0, r.stream>>>(r.x, count,
                                                                                       reinterpret_cast<__half*>(r.xrec));
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 grid(static_cast<unsigned>((r.n + kTcM - 1) / kTcM), static_cast<unsigned>((r.batch + kTcN - 1) / kTcN),
                  static_cast<unsigned>(splits));
  gemm_tc<Q><<<grid, kTcThreads, smem, r.stream>>>(wmap, xmap, p);
  e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  const int64_t ycount = static_cast<int64_t>(r.batch) * r.n;
  int64_t blocks = (ycount + 255) / 256;
  if (blocks > static_cast<int64_t>(r.sms) * 8) blocks = static_cast<int64_t>(r.sms) * 8;
  tc_reduce<<<static_cast<unsigned>(blocks), 256, 0, r.stream>>>(p.ws, splits, ycount, r.y);
  return cudaGetLastError();
}

// Bounded wait until every rank's flag in `flags` has reached this rank's
// epoch for the group (the epoch its last fused GEMV published).
static __global__ void __launch_bounds__(32) gather_wait_kernel(const uint32_t* flags, int world,
                                                               const uint32_t* epoch, uint32_t* status) {
  const int r = threadIdx.x;
  if (r >= world) return;
  const uint32_t e = *epoch;
  const uint64_t t0 = global_ns();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
    if (static_cast<int32_t>(v - e) >= 0) break;
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(status, kStatusGatherTimeout);
      break;
    }
  }
}

inline cudaError_t launch_gather_wait(const uint32_t* flags, int world, const uint32_t* epoch, uint32_t* status,
                                      cudaStream_t stream) {
  gather_wait_kernel<<<1, 32, 0, stream>>>(flags, world, epoch, status);
  return cudaGetLastError();
}

// Batch-1 tensor-core kernel (gemv_tc1, Q4_K).  Compute warps = super-blocks
// per chunk: the whole row when it has at most 16 super-blocks, else the
// largest divisor of the row's super-blocks in [8, 16], else 16.  The
// activation fragments of as many whole chunks as leave room for 4 stages
// (else 3, else 2) are held at a time (a part of k); then as many stages as
// fit, up to 8.
struct Tc1Config {
  int nw = 0, mt = 1, nch = 0, stride = 0, stage_bytes = 0, nst = 0, part_chunks = 0, rows_max = 0;
  int builders = 0;  // rows in several parts of k: builder warps, two fragment buffers
  int split = 1;     // rows in several parts of k: CTAs per cluster, one part each
  int ranges = 0;    // split: row ranges (clusters) wanted
  size_t smem = 0;
};
constexpr int kTc1MaxSplit = 8;  // portable cluster size

// MMA tiles per warp of a batch-1 tensor-core launch (a row group is 16 rows
// per tile).  Two, measured on B200 against one (twice the warps, 16-row
// groups): Llama-3-70B gate+up 65.8 against 70.3 us, the Qwen2-7B layer step
// 58.6 against 66.3 us; the per-tile and per-row-group work of a warp is
// shared by twice the weights and the B fragments by both tiles.
inline int tc1_mt_for(int k) {
  (void)k;
  const int forced = tuning().tc_mt;
  if (forced == 1 || forced == 2) return forced;
  return 2;
}

// CTAs of a batch-1 tensor-core launch of n rows: one per SM and one
// two-tile row group (32 rows) each at least; but where that leaves more
// than half the SMs idle, one 16-row MMA tile each (a row group of at most
// 16 rows converts one tile, half the work): Llama-3-70B o and down
// row-sharded over 8 GPUs, 1024 rows, run on 64 CTAs instead of 32.  A
// row's arithmetic does not depend on its CTA or on its group's tiles.
// Measured on B200 (Q4_K, us, 32-row / 16-row CTAs, bit-identical y):
// 1024 x 8192 8.73 / 6.99, 2048 x 8192 9.08 / 7.46, 1024 x 28672 23.95 /
// 18.63, 2048 x 28672 24.35 / 19.54, 512 x 3584 5.22 / 4.88; where 32-row
// CTAs already cover more than half the SMs the extra CTAs cost a little
// (3584 x 3584 7.45 / 7.64, 4096 x 28672 25.05 / 25.75).
inline int tc1_grid(int64_t n, int sms) {
  int64_t g = (n + 2 * kTc1Rows - 1) / (2 * kTc1Rows);
  if (2 * g <= sms) g = (n + kTc1Rows - 1) / kTc1Rows;
  if (g > sms) g = sms;
  return g < 1 ? 1 : static_cast<int>(g);
}

// Row ranges (clusters of s CTAs, one per s SMs) of a split launch of n
// rows, sized as tc1_grid sizes CTAs; and the most rows one range may hold,
// allowing for as few as half of those clusters resident at once (the launch
// runs no more ranges than the device holds clusters).
inline int tc1_split_ranges(int64_t n, int sms, int s) { return tc1_grid(n, sms / s > 0 ? sms / s : 1); }
inline int tc1_split_rows(int64_t n, int sms, int s) {
  const int t = tc1_split_ranges(n, sms, s);
  const int lo = t / 2 > 0 ? t / 2 : 1;
  return static_cast<int>((n + lo - 1) / lo);
}

// swiglu: x is read as silu(x) * x_mul (the down projection's SwiGLU),
// whose exponentials the 64 threads of the builder warps would form more
// slowly than the compute warps (Qwen2-7B decode token: 2.85 ms with
// builders against 2.79 without).
inline bool tc1_config(int ts, int k, int64_t n, int sms, bool long_rows, bool swiglu, Tc1Config* c) {
  if (k % 256 != 0 || k <= 0 || sms < 1) return false;
  const int sbs = k / 256;
  const int mt = tc1_mt_for(k);
  // compute warps: one super-block each per chunk; two MMA tiles per warp
  // use half as many warps for the same tile bytes
  const int maxw = mt == 2 ? 8 : kTc1MaxWarps;
  int nw = 0;
  if (sbs <= maxw) {
    nw = sbs;
  } else {
    for (int d = maxw; d >= maxw / 2 && !nw; --d)
      if (sbs % d == 0) nw = d;
    if (!nw) nw = maxw;
  }
  const int grid = tc1_grid(n, sms);
  const int64_t rows_max = (n + grid - 1) / grid;
  if (rows_max > (1 << 20)) return false;
  c->rows_max = static_cast<int>(rows_max);
  const int budget = tuned(tuning().smem_bytes, kSmemBudget);
  const int want = tuned(tuning().tc_stages, 3);
  // two tiles per warp: 11 compute warps (three warps per SM sub-partition
  // with the producer) where the chunks waste at most one super-block each
  // and the whole row's fragments leave room for `want` stages.  Measured on
  // B200 (Llama-3-70B, k = 8192, 3 chunks of 11, 11 and 10 super-blocks):
  // gate+up 61.3 us against 64.2 with 8 warps (4 chunks of 8), q+k+v 18.5
  // against 19.1; 9 or 10 warps (4 chunks) 69.6-72.9.
  if (mt == 2 && sbs > kTc1MaxWarpsMt2) {
    const int w = kTc1MaxWarpsMt2, ch = (sbs + w - 1) / w;
    const int st = round_up(kTc1Rows * mt * tc1_row_stride(w, ts), 128);
    if (ch * w - sbs <= ch && tc1_layout(want, ch * w, c->rows_max, st).total <= budget) nw = w;
  }
  const int forced = tuning().nwarps;
  if (forced >= 1 && forced <= (mt == 2 ? kTc1MaxWarpsMt2 : maxw)) nw = forced;
  c->nw = nw;
  c->mt = mt;
  c->nch = (sbs + nw - 1) / nw;
  c->stride = tc1_row_stride(nw, ts);
  c->stage_bytes = round_up(kTc1Rows * mt * c->stride, 128);
  // the whole row's fragments if they leave room for `want` stages, else
  // parts of k: with two tiles per warp two builder warps fill one fragment
  // buffer while the compute warps read the other, and each buffer holds as
  // many whole chunks as leave room for `want` stages (else fewer, down to
  // 2).  Measured on B200 (down projections, us): Llama-3-70B k = 28672
  // 41.6 at 3 stages x 4 parts, 41.7 at 4 x 5, 45.7 at 2 x 7 (one builder
  // warp 44.2, none 47.2 on the CUDA-core kernel); Qwen2-7B k = 18944 17.1 at
  // 3 x 3, 18.1 at 4 x 4, 18.9 at 2 x 2 without builders.
  int pc = 0, builders = 0, split = 1;
  if (tc1_layout(want, c->nch * nw, c->rows_max, c->stage_bytes).total <= budget) {
    pc = c->nch;
  } else if (tuned(tuning().tc_split, 1) && sms >= 2) {
    // a cluster of s CTAs per row range, CTA r building and streaming part r
    // of k only: the fewest parts whose fragments leave room for `want`
    // stages (else fewer), balanced in chunks.  Each part's row sums are
    // formed as in a one-CTA launch and cluster rank 0 adds them in part
    // order, so y does not depend on n or on the grid.  Measured on B200
    // (Q4_K, us, one CTA per range with builder warps / clusters of two):
    // 8192 x 28672 42.9 / 39.5, 2048 x 28672 24.5 / 15.7, 1024 x 28672
    // 24.0 / 12.7; where the row ranges are as many either way a little
    // slower (4096 x 28672 25.1 / 25.6, 3584 x 18944 18.1 / 18.3).
    for (int w = want; w >= 2 && split == 1; --w) {
      for (int s = 2; s <= kTc1MaxSplit && s <= sms; ++s) {
        const int q = (c->nch + s - 1) / s;
        if ((c->nch + q - 1) / q != s) continue;  // s parts of q chunks would leave one empty
        if (tc1_layout(w, q * nw, tc1_split_rows(n, sms, s), c->stage_bytes).total <= budget) {
          pc = q;
          split = s;
          break;
        }
      }
    }
  }
  if (!pc) {
    builders = mt == 2 && nw <= 8 && !swiglu ? tuned(tuning().tc_builders, 2) : 0;
    if (builders > 2) builders = 2;
    const int nbuf = builders ? 2 : 1;
    const int forced_pc = tuning().tc_part_chunks;
    if (forced_pc >= 1 && forced_pc < c->nch) {
      pc = forced_pc;
    } else {
      for (int w = want; w >= 2 && !pc; --w) {
        for (int q = c->nch - 1; q >= 1; --q) {
          if (tc1_layout(w, q * nw, c->rows_max, c->stage_bytes, nbuf).total <= budget) {
            pc = q;
            break;
          }
        }
      }
    }
  }
  if (!pc) return false;
  if (split > 1) {
    c->rows_max = tc1_split_rows(n, sms, split);
    c->ranges = tc1_split_ranges(n, sms, split);
  }
  // rows longer than one part of k in one CTA: with builder warps the parts'
  // fragments are built behind the compute; without them they are rebuilt
  // while the ring drains, which measured on B200 behind the CUDA-core
  // kernel at three parts (Llama-3-70B down, k = 28672: 50.8 against 47.1
  // us), so rows of more than two parts without builders stay on it unless
  // long_rows (FRC_OPT_BATCH1_TC = 2)
  if (split == 1 && !builders && (c->nch + pc - 1) / pc > 2 && !long_rows) return false;
  const int nbuf = builders ? 2 : 1;
  const int forced_nst = tuning().nstage;
  int nst = forced_nst > 0 ? forced_nst : 8;
  for (; nst >= 2; --nst)
    if (tc1_layout(nst, pc * nw, c->rows_max, c->stage_bytes, nbuf).total <= budget) break;
  if (nst < 2) return false;
  c->part_chunks = pc;
  c->builders = builders;
  c->split = split;
  c->nst = nst;
  c->smem = static_cast<size_t>(tc1_layout(nst, pc * nw, c->rows_max, c->stage_bytes, nbuf).total);
  return true;
}

template <int Q>
inline cudaError_t launch_tc1(GemvParams p, const GemvRequest& r, const Tc1Config& c) {
  p.tc_kc = c.nw;
  p.tc_nchunk = c.nch;
  p.tc_stride = c.stride;
  p.tc_bias = kH2Bias;
  p.tc_part_chunks = c.part_chunks;
  p.tc_rows_max = c.rows_max;
  p.tc_rg = kTc1Rows * c.mt;
  p.stage_stride = c.stage_bytes;
  p.nstage = c.nst;
  p.tc_split = c.split;
  if (c.split > 1 && (c.builders || c.mt != 2 || c.nw > 8)) return cudaErrorInvalidValue;  // not a split form
  const int threads = (c.nw + 1 + c.builders) * 32;
  // two MMA tiles per warp: up to 8 compute warps (+ builder warps for rows
  // in parts of k); one: up to 15 compute warps run the 16-warp
  // instantiation (128 registers), 16 the 17-warp one
  auto kernel = c.mt == 2 ? (c.builders == 2   ? gemv_tc1<Q, 8, 2, 2>
                             : c.builders == 1 ? gemv_tc1<Q, 8, 2, 1>
                             : c.nw > 8        ? gemv_tc1<Q, kTc1MaxWarpsMt2, 2, 0>
                                               : gemv_tc1<Q, 8, 2, 0>)
                          : (c.nw < kTc1MaxWarps ? gemv_tc1<Q, kTc1MaxWarps - 1, 1, 0>
                                                 : gemv_tc1<Q, kTc1MaxWarps, 1, 0>);
  int per_sm = 0;
  cudaError_t e = kernel_occupancy(reinterpret_cast<const void*>(kernel), r.device, threads, c.smem, &per_sm);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  // one tensor map per matrix: [rows][super-blocks][TS / 8 words of 8 bytes]
  constexpr int TS = Fmt<Q>::TS;
  Tc1Maps maps;
  std::memset(&maps, 0, sizeof(maps));
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  const int sbs = p.k / 256;
  for (int m = 0; m < p.nmat; ++m) {
    const int64_t rows = p.mat_end[m] - (m ? p.mat_end[m - 1] : 0);
    const cuuint64_t dims[3] = {TS / 8, static_cast<cuuint64_t>(sbs), static_cast<cuuint64_t>(rows > 0 ? rows : 1)};
    const cuuint64_t strides[2] = {TS, static_cast<cuuint64_t>(p.row_bytes)};
    const cuuint32_t estr[3] = {1, 1, 1};
    for (int b = 0; b < kTc1Boxes; ++b) {
      const cuuint32_t box[3] = {TS / 8, static_cast<cuuint32_t>(c.nw), static_cast<cuuint32_t>(kTc1MaxRows >> b)};
      if (encode(&maps.m[m][b], CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<uint8_t*>(p.mat_w[m]), dims, strides,
                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(tc1_grid(p.n, r.sms)));
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = c.smem;
  cfg.stream = r.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = tuned(tuning().pdl, 1) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (c.split > 1) {
    // clusters of c.split CTAs along x, as many row ranges as the device
    // holds clusters at once (at least the half tc1_config sized rows for)
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(c.split);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    cfg.gridDim = dim3(static_cast<unsigned>(c.split * c.ranges));
    int clusters = 0;
    e = max_active_clusters(reinterpret_cast<const void*>(kernel), r.device, cfg, &clusters);
    if (e != cudaSuccess) return e;
    const int ranges = c.ranges < clusters ? c.ranges : clusters;
    if (ranges < 1 || (p.n + ranges - 1) / ranges > c.rows_max) return cudaErrorInvalidConfiguration;
    cfg.gridDim = dim3(static_cast<unsigned>(c.split * ranges));
  }
  return cudaLaunchKernelEx(&cfg, kernel, maps, p);
}

// Largest tile footprint must fit in shared memory with two stages.
template <int Q>
inline bool tiles_fit(int row_bytes) {
  return 2 * (2 * row_bytes + 32) + 4096 <= 200 * 1024;
}

template <int Q>
cudaError_t launch_gemv(const GemvRequest& r) {
  using F = Fmt<Q>;
  GemvParams p{};
  p.w = r.w;
  p.x = r.x;
  p.y = r.y;
  p.n = r.n;
  p.k = r.k;
  p.batch = r.batch;
  p.row_bytes = (r.k / F::QK) * F::TS;
  p.units = (r.k / F::QK) * F::UPB;
  p.status = r.status;
  if (r.nmat > 1) {
    p.nmat = r.nmat;
    int64_t end = 0;
    for (int m = 0; m < r.nmat; ++m) {
      end += r.mat_n[m];
      p.mat_end[m] = end;
      p.mat_w[m] = r.mat_w[m];
      p.mat_y[m] = r.mat_y[m];
    }
    p.n = end;
  } else {
    p.nmat = 1;
    p.mat_end[0] = r.n;
    p.mat_w[0] = r.w;
    p.mat_y[0] = r.y;
  }
  if (!tiles_fit<Q>(p.row_bytes)) return cudaErrorInvalidValue;
  if (r.g_world > 1) {
    p.g_world = r.g_world;
    p.g_rank = r.g_rank;
    p.g_ybase = r.g_ybase;
    for (int i = 0; i < r.g_world; ++i) {
      p.g_peer_y[i] = r.g_peer_y[i];
      p.g_flags[i] = r.g_flags[i];
    }
    p.g_done = r.g_done;
    p.g_epoch = r.g_epoch;
  }
  if (r.w_world > 1) {
    p.w_world = r.w_world;
    p.w_flags = r.w_flags;
    p.w_epoch = r.w_epoch;
  }
  const bool exact_batched = opt(options().batched_fp32) != 0;
  if ((r.x_mul || r.y_accum || r.x_norm_w) && (r.batch != 1 || r.g_world > 1 || opt(options().batch1_int16)))
    return cudaErrorNotSupported;  // only the batch-1 fp32-activation kernel has them
  p.x_mul = r.x_mul;
  p.y_accum = r.y_accum;
  p.x_norm_w = r.x_norm_w;
  p.x_norm_eps = r.x_norm_eps;
  if (r.batch == 1) {
    GemvParams b1 = p;
    b1.units = (r.k / F::QK) * I8<Q>::UPB;
    if constexpr (Q == kQ4_K || Q == kQ5_K) {
      Tc1Config c;
      if (!opt(options().batch1_int16) && opt(options().batch1_tc) &&
          tc1_config(Fmt<Q>::TS, r.k, b1.n, r.sms, opt(options().batch1_tc) == 2, r.x_mul != nullptr, &c))
        return launch_tc1<Q>(b1, r, c);
    }
    const cudaError_t e =
        opt(options().batch1_int16) ? launch_b1_any<Q, false>(b1, r) : launch_b1_any<Q, true>(b1, r);
    if (e != cudaErrorInvalidValue) return e;
    (void)cudaGetLastError();
    // a row longer than one CTA's threads cover: the column-reusing kernel
    // (fp32 activations), without the fused multi-matrix, gather, SwiGLU or
    // accumulating forms
    if (r.nmat > 1 || r.g_world > 1 || r.w_world > 1 || r.x_mul || r.y_accum || r.x_norm_w)
      return cudaErrorNotSupported;
    return launch_xb<Q, 4>(p, r);
  }
  // the fused multi-matrix launch and the fused all-gather exist only in the
  // batch-1 kernel: callers fall back (per matrix / NCCL)
  if (r.nmat > 1 || r.g_world > 1 || r.w_world > 1) return cudaErrorNotSupported;
  if (r.xrec && !exact_batched) return launch_mma<Q>(r);
  if (r.batch <= 4) return launch_xb<Q, 4>(p, r);
  if (r.batch <= 8) return launch_xb<Q, 8>(p, r);
  return launch_xb<Q, 16>(p, r);
}

// ---------------------------------------------------------------------------
// Bit-exact dequantisation: thread i writes elements [4i, 4i+4).
// ---------------------------------------------------------------------------
template <int Q>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ w, int64_t n_elems,
                                                     float* __restrict__ out) {
  using F = Fmt<Q>;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
  for (int64_t e0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; e0 < n_elems;
       e0 += stride) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t e = e0 + i;
      if (e < n_elems) {
        const int64_t b = e / F::QK;
        out[e] = dequant_elem<Q>(w + b * F::TS, static_cast<int>(e - b * F::QK));
      }
    }
  }
}

template <int Q>
cudaError_t launch_dequant(const DequantRequest& r) {
  if (r.n_elems <= 0) return cudaSuccess;
  const int64_t threads_needed = (r.n_elems + 3) / 4;
  int64_t grid = (threads_needed + 255) / 256;
  const int64_t cap = static_cast<int64_t>(r.sms) * 16;
  if (grid > cap) grid = cap;
  dequant_kernel<Q><<<static_cast<unsigned>(grid), 256, 0, r.stream>>>(r.w, r.n_elems, r.out);
  return cudaGetLastError();
}

}  // namespace frc
