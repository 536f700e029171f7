// Fused dequantise + GEMV kernels for GGUF row-major weights.
//
// gemv_b1 (batch 1, the decode path) streams weight rows through shared
// memory in independent per-slot pipelines (described above the kernel).  Its
// activation arithmetic is a template parameter: exact fp32 activations and
// fp32 products (units_f32.cuh, the reference's arithmetic and the default),
// or activations on a 16-bit integer grid with dp4a products
// (units_dp4a.cuh, opt-in).
//
// gemv_xb (batch 2..16, exact fp32 activations) is persistent and
// warp-specialised: the last warp is the producer (one lane streams tiles of
// RT consecutive rows into a ring of shared-memory stages with cp.async.bulk,
// signalling each stage's mbarrier), the others are consumers; consumer
// thread t owns the units t, t + NCT, ... of every row, decodes each unit once
// per row and reuses it for every activation column (read through L1).
//
// Each CTA owns the contiguous rows [c*n/G, (c+1)*n/G), which balances work
// to within one row; a tile's global start is rounded down to 16 bytes for
// the bulk copy (its offset is kept in shared memory), and the <16-byte tail
// of the last tile is copied by the issuing thread.  Per-row partial sums are
// reduced with a register-transpose butterfly (V-1 shuffles for V rows), then
// across warps through shared memory.  Every mbarrier wait is bounded by
// wall-clock time (kWaitLimitNs, read from %globaltimer); on a timeout the CTA
// raises a shared abort flag, records a status bit, stops computing and still
// passes every barrier, so it always exits.
#pragma once

#include <type_traits>

#include "formats.cuh"
#include "units_dp4a.cuh"
#include "units_f32.cuh"

namespace frc {

constexpr int kMaxConsumerWarps = 15;  // + 1 producer = 512 threads, 128 registers each
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait
constexpr int kMaxGatherRanks = 8;

struct GemvParams {
  const uint8_t* w;   // raw blocks, 16-byte aligned
  const float* x;     // (batch, k)
  float* y;           // (batch, n)
  int64_t n;          // rows
  int k;              // columns
  int batch;
  int row_bytes;      // (k / QK) * TS
  int units;          // units per row
  int stage_stride;   // bytes per shared-memory stage
  int nstage;
  int wps;            // gemv_b1: warps per slot (one slot covers one row's units)
  int pre_stages;     // gemv_b1: stages per slot filled before the grid dependency wait
  uint32_t* status;   // device status word
  // gemv_b1 row space: nmat matrices sharing x and k, rows concatenated;
  // matrix m covers rows [mat_end[m-1], mat_end[m]) of the n rows
  int nmat;
  int64_t mat_end[4];
  const uint8_t* mat_w[4];  // each 16-byte aligned
  float* mat_y[4];
  // gemv_b1 fused all-gather (g_world > 1): every y value is also stored at
  // the same offset from g_peer_y[r] as from g_ybase, for each rank r (the
  // rank's shard in r's gathered buffer, over NVLink for r != this rank);
  // the last slot of the grid to finish publishes the group's next epoch in
  // every rank's flag array (slot g_rank)
  int g_world, g_rank;
  const float* g_ybase;
  float* g_peer_y[kMaxGatherRanks];
  uint32_t* g_flags[kMaxGatherRanks];
  uint32_t* g_done;   // slots finished in this launch (reset by the last)
  uint32_t* g_epoch;  // gathers completed by this rank
  // gemv_b1: before reading x, wait until every rank has published the
  // epoch of an earlier fused gather (w_world > 1): x may be its output
  int w_world;
  const uint32_t* w_flags;
  const uint32_t* w_epoch;
  // gemv_b1 with fp32 activations: x_mul != null reads the activations as
  // silu(x) * x_mul (the SwiGLU of a gate and an up projection feeding down);
  // y_accum adds to y instead of storing (a residual stream)
  const float* x_mul;
  int y_accum;
  // gemv_b1 with fp32 activations: x_norm_w != null reads the activations
  // as RMSNorm(x) * x_norm_w (eps x_norm_eps), the norm of the whole row of x
  // formed inside every slot
  const float* x_norm_w;
  float x_norm_eps;
  // gemv_tc1: super-blocks per chunk (= compute warps), chunks per row, the
  // row stride of a stage in bytes, and the fp16 pair 1024, 1024 (0x64006400;
  // a parameter, so the mask-and-or of a quant word is one instruction with
  // the pair as its register operand)
  int tc_kc, tc_nchunk, tc_stride;
  uint32_t tc_bias;
  // gemv_tc1: chunks per part of k (the activation fragments a CTA holds at
  // a time) and the most rows one CTA owns
  int tc_part_chunks, tc_rows_max;
  int tc_rg;  // gemv_tc1: rows per row group (16 per MMA tile of a warp)
  // gemv_tc1: CTAs per cluster.  1: each CTA owns a row range and every part
  // of k; s > 1: the s CTAs of a cluster share a row range, CTA r computing
  // part r of k, and cluster rank 0 adds the parts' row sums in order
  int tc_split;
};

constexpr int kMaxMats = 4;

FRC_DEVICE_INLINE uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase that also gives up as soon as another
// thread of the CTA has raised `abort`.
FRC_DEVICE_INLINE bool wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      return false;
    }
  }
}

// Sum V per-lane values across the warp.  Afterwards lane l holds the total of
// value index (l >> (5 - log2 V)) for V <= 32; V > 32 is done in 32-chunks and
// lane l holds chunk c's value (c*32 + l) in out[c].
template <int V>
FRC_DEVICE_INLINE void butterfly(float (&v)[V], int lane) {
  static_assert((V & (V - 1)) == 0 && V >= 1 && V <= 32, "V must be a power of two <= 32");
  int width = V;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (width > 1) {
      const bool upper = (lane & o) != 0;
      const int h = width / 2;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < h) {
          const float send = upper ? v[i] : v[i + h];
          const float keep = upper ? v[i + h] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      width = h;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
}

struct SmemLayout {
  uint64_t* full;
  uint64_t* empty;
  int* abort;
  float* red;       // [2][kMaxConsumerWarps][VMAX]
  uint8_t* stages;  // nstage * stage_stride
};

template <int VMAX>
FRC_DEVICE_INLINE SmemLayout carve(uint8_t* smem, int nstage) {
  SmemLayout L;
  L.full = reinterpret_cast<uint64_t*>(smem);
  L.empty = L.full + nstage;
  L.abort = reinterpret_cast<int*>(L.empty + nstage);
  L.red = reinterpret_cast<float*>(smem + 256);
  const int red_bytes = 2 * kMaxConsumerWarps * VMAX * 4;
  L.stages = smem + ((256 + red_bytes + 127) / 128) * 128;
  return L;
}

template <int VMAX>
__host__ __device__ constexpr int smem_header_bytes() {
  return ((256 + 2 * kMaxConsumerWarps * VMAX * 4 + 127) / 128) * 128;
}

// Producer lane: stream the tiles of rows [r0, r1) in chunks of RT rows.
FRC_DEVICE_INLINE void produce(const GemvParams& p, const SmemLayout& L, int64_t r0, int64_t r1, int RT) {
  volatile int* abort = L.abort;
  int issued = 0;
  for (int64_t t0 = r0; t0 < r1; t0 += RT, ++issued) {
    const int s = issued % p.nstage;
    const uint32_t ph = static_cast<uint32_t>(issued / p.nstage) & 1u;
    if (!wait_phase(&L.empty[s], ph ^ 1u, abort)) {
      atomicOr(p.status, kStatusEmptyWaitTimeout);
      break;
    }
    const int64_t t1 = t0 + RT < r1 ? t0 + RT : r1;
    const uint64_t gs = static_cast<uint64_t>(t0) * p.row_bytes;
    const uint64_t ge = static_cast<uint64_t>(t1) * p.row_bytes;
    const uint64_t a0 = gs & ~uint64_t(15), a1 = ge & ~uint64_t(15);
    uint8_t* dst = L.stages + static_cast<size_t>(s) * p.stage_stride;
    for (uint64_t b = a1; b < ge; ++b) dst[b - a0] = p.w[b];
    const uint32_t bulk = static_cast<uint32_t>(a1 - a0);
    mbar_arrive_expect_tx(&L.full[s], bulk);
    if (bulk) bulk_g2s(dst, p.w + a0, bulk, &L.full[s]);
  }
  // Every issued copy lands before this lane (and so the CTA) exits.
  const int first = issued > p.nstage ? issued - p.nstage : 0;
  for (int i = first; i < issued; ++i) {
    if (!wait_phase(&L.full[i % p.nstage], static_cast<uint32_t>(i / p.nstage) & 1u, abort)) {
      // the abort flag may stop this wait early; give in-flight copies a
      // second bounded chance that ignores the flag
      int zero = 0;
      if (!wait_phase(&L.full[i % p.nstage], static_cast<uint32_t>(i / p.nstage) & 1u, &zero)) {
        atomicOr(p.status, kStatusDrainTimeout);
      }
    }
  }
}

FRC_DEVICE_INLINE void cta_rows(int64_t n, int64_t& r0, int64_t& r1) {
  r0 = static_cast<int64_t>(blockIdx.x) * n / gridDim.x;
  r1 = static_cast<int64_t>(blockIdx.x + 1) * n / gridDim.x;
}

FRC_DEVICE_INLINE void load_run16(const float* src, float* dst) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = __ldg(s4 + i);
    dst[4 * i] = v.x;
    dst[4 * i + 1] = v.y;
    dst[4 * i + 2] = v.z;
    dst[4 * i + 3] = v.w;
  }
}

// ---------------------------------------------------------------------------
// batch 1: gemv_b1<Q, UPT, RPS, F32>
//
// F32 = true: every thread keeps its units' fp32 activations in registers
// (UnitXF, loaded straight from global memory) and UnitDotF32 multiplies them
// with the decoded quants in fp32.  F32 = false: each CTA quantises x once into
// shared-memory records on a 16-bit integer grid (quantise_words), each thread
// copies its units' records into registers (UnitX) and UnitDotI8 runs dp4a.
//
// Every warp of the CTA computes; there is no producer warp.  The warps form
// slots of p.wps warps, and each slot is an independent pipeline: it owns a
// contiguous share of the CTA's rows, its own ring of p.nstage shared-memory
// stages (RPS rows each) and its own mbarriers.  Thread st of a slot owns
// units st, st + 32 wps, ... of every row.  Per tile: wait for the stage,
// accumulate, reduce across the slot, pass the slot's named barrier, and then
// the slot leader refills that stage with the tile NSTAGE ahead (every thread
// of the slot has finished reading it) while the first RPS threads write y.
// ---------------------------------------------------------------------------
FRC_DEVICE_INLINE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Issue the bulk copy of rows [l0, l1) of the matrix at `w` into `dst` (a
// stage), with the <16-byte tail copied by this thread; completion on `bar`.
FRC_DEVICE_INLINE void issue_tile(const GemvParams& p, const uint8_t* w, uint8_t* dst, uint64_t* bar, int64_t l0,
                                  int64_t l1) {
  const uint64_t gs = static_cast<uint64_t>(l0) * p.row_bytes;
  const uint64_t ge = static_cast<uint64_t>(l1) * p.row_bytes;
  const uint64_t a0 = gs & ~uint64_t(15), a1 = ge & ~uint64_t(15);
  for (uint64_t b = a1; b < ge; ++b) dst[b - a0] = w[b];
  const uint32_t bulk = static_cast<uint32_t>(a1 - a0);
  mbar_arrive_expect_tx(bar, bulk);
  if (bulk) bulk_g2s(dst, w + a0, bulk, bar);
}

// A tile of at most `rps` rows starting at global row t0, clipped to the end of
// its matrix and to r1.
struct Tile {
  int64_t t1;     // global end row
  int64_t local;  // first row inside matrix m
  int m;
};

FRC_DEVICE_INLINE Tile tile_at(const GemvParams& p, int64_t t0, int64_t r1, int rps) {
  int m = 0;
  while (m + 1 < p.nmat && t0 >= p.mat_end[m]) ++m;
  const int64_t start = m ? p.mat_end[m - 1] : 0;
  int64_t end = p.mat_end[m] < r1 ? p.mat_end[m] : r1;
  Tile t;
  t.t1 = t0 + rps < end ? t0 + rps : end;
  t.local = t0 - start;
  t.m = m;
  return t;
}

FRC_DEVICE_INLINE int count_tiles(const GemvParams& p, int64_t r0, int64_t r1, int rps) {
  int n = 0;
  int64_t start = 0;
  for (int m = 0; m < p.nmat; ++m) {
    const int64_t a = r0 > start ? r0 : start;
    const int64_t b = r1 < p.mat_end[m] ? r1 : p.mat_end[m];
    if (b > a) n += static_cast<int>((b - a + rps - 1) / rps);
    start = p.mat_end[m];
  }
  return n;
}

// Warps per CTA at most, from the activation registers a thread holds (UPT
// units of 2 E/4 + NG + 1 words on the integer grid, E + NG in fp32): 16 warps
// (128 registers each) up to 72 activation registers, 12 warps (168
// registers) beyond.  One fp32 K-quant unit (66 registers) fits the 128
// (ptxas: no spills for Q4_K, Q6_K, Q8_0, Q1_0; a few bytes for Q5_K at
// four- and eight-row tiles).
template <int Q, int UPT, bool F32>
__host__ __device__ constexpr int b1_max_warps() {
  return UPT * (F32 ? I8<Q>::E + I8<Q>::NG : 2 * I8<Q>::E / 4 + I8<Q>::NG + 1) <= 72 ? 16 : 12;
}

FRC_DEVICE_INLINE void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FRC_DEVICE_INLINE void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Stores one y value locally and, with a fused all-gather, into every rank's
// gathered buffer.
FRC_DEVICE_INLINE void put_y(const GemvParams& p, int g_world, float* dst, float v) {
  if (p.y_accum) v += *dst;
  *dst = v;
  if (g_world > 1) {
    const int64_t off = dst - p.g_ybase;
    for (int r = 0; r < g_world; ++r) p.g_peer_y[r][off] = v;
  }
}

// A relaxed system-scope store; after one fence.sc.sys it completes a
// release pattern (the fence orders every earlier write before it).
FRC_DEVICE_INLINE void st_relaxed_sys(uint32_t* ptr, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// Called by one thread per slot after the slot barrier that follows the
// slot's y stores: the slot's stores are released at GPU scope before its
// arrival; the last slot of the grid acquires them through the counter and
// publishes the next epoch to every rank after one system-scope fence
// (fences are cumulative, so it covers every slot's stores, remote ones
// included).
FRC_DEVICE_INLINE void gather_arrive(const GemvParams& p, int g_world, int slots) {
  if (g_world <= 1) return;
  __threadfence();
  const uint32_t total = gridDim.x * static_cast<uint32_t>(slots);
  if (atomicAdd(p.g_done, 1u) + 1u == total) {
    __threadfence();
    __threadfence_system();
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(p.g_epoch) + 1u;
    for (int r = 0; r < p.g_world; ++r) st_relaxed_sys(p.g_flags[r] + p.g_rank, e);
    *p.g_epoch = e;
    *p.g_done = 0u;
  }
}

template <int Q, bool F32, typename XU>
FRC_DEVICE_INLINE float unit_dot(uint32_t row, const UnitCtx& c, const XU& x) {
  if constexpr (F32) {
    return UnitDotF32<Q>::dot(row, c, x);
  } else {
    return UnitDotI8<Q>::dot(row, c, x);
  }
}

template <int Q, int UPT, int RPS, bool F32>
__global__ void __launch_bounds__(b1_max_warps<Q, UPT, F32>() * 32, 1) gemv_b1(GemvParams p) {
  constexpr int RW = F32 ? 0 : record_words<Q>();
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = static_cast<int>(blockDim.x >> 5);
  const int slots = nwarps / p.wps;
  const int nst = p.nstage;
  // layout: full[slots][nst] | abort | red[slots][2][wps][RPS] | records | stages
  uint64_t* full_all = reinterpret_cast<uint64_t*>(smem);
  int* abort_flag = reinterpret_cast<int*>(full_all + slots * nst);
  float* red_all = reinterpret_cast<float*>(smem + ((slots * nst * 8 + 4 + 15) / 16) * 16);
  const int red_bytes = slots * 2 * p.wps * RPS * 4;
  uint32_t* records = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(red_all) + ((red_bytes + 15) / 16) * 16);
  uint8_t* stage_all = reinterpret_cast<uint8_t*>(records + p.units * RW);
  stage_all = smem + ((stage_all - smem + 127) / 128) * 128;

  if (threadIdx.x == 0) {
    for (int i = 0; i < slots * nst; ++i) mbar_init(&full_all[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  const int slot = warp / p.wps;
  const int st = threadIdx.x - slot * p.wps * 32;
  const int spt = p.wps * 32;
  uint64_t* full = full_all + slot * nst;
  uint8_t* stages = stage_all + static_cast<size_t>(slot) * nst * p.stage_stride;
  float* red = red_all + slot * 2 * p.wps * RPS;
  volatile int* abort = abort_flag;

  // rows of this slot
  int64_t c0, c1;
  cta_rows(p.n, c0, c1);
  const int64_t r0 = c0 + (c1 - c0) * slot / slots;
  const int64_t r1 = c0 + (c1 - c0) * (slot + 1) / slots;
  const int ntiles = slot < slots ? count_tiles(p, r0, r1, RPS) : 0;

  // The weights are never written by another kernel: start streaming them
  // before waiting for the previous kernel in the stream (programmatic
  // dependent launch), which may still be producing x.
  int issued = 0;  // tiles handed to the copy engine (leader only)
  const int leader = p.wps == 1 ? 0 : spt - 32;  // lane 0 of the slot's last warp
  int64_t next_issue = r0;  // leader's cursor over the slot's tiles
  if (st == leader && ntiles > 0) {
    for (int i = 0; i < p.pre_stages && i < nst && i < ntiles; ++i, ++issued) {
      const Tile t = tile_at(p, next_issue, r1, RPS);
      issue_tile(p, p.mat_w[t.m], stages + static_cast<size_t>(i) * p.stage_stride, &full[i], t.local,
                 t.local + (t.t1 - next_issue));
      next_issue = t.t1;
    }
  }
  griddep_wait();
  griddep_launch_dependents();
  // ranks this launch's outputs go to: after a gather wait that ran out, a
  // peer may still be reading its buffer, so this launch stores locally only
  // and publishes nothing (the status bit tells the caller the step is void)
  int g_world = p.g_world;
  if (p.w_world > 1) {  // an earlier fused gather must be complete on every rank
    if (threadIdx.x < static_cast<unsigned>(p.w_world)) {
      const uint32_t e = *p.w_epoch;
      const uint64_t t0 = global_ns();
      while (true) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.w_flags + threadIdx.x) : "memory");
        if (static_cast<int32_t>(v - e) >= 0) break;
        if (global_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.status, kStatusGatherTimeout);
          *abort_flag = 2;  // read below; the tile loop only tests for nonzero after this point
          break;
        }
      }
    }
    __syncthreads();
    if (*abort_flag == 2) {
      g_world = 1;
      __syncthreads();  // every thread has read the flag
      if (threadIdx.x == 0) *abort_flag = 0;
      __syncthreads();
    }
  }

  UnitCtx cx[UPT];
  bool uval[UPT];
#pragma unroll
  for (int i = 0; i < UPT; ++i) {
    const int u = st + i * spt;
    uval[i] = u < p.units;
    cx[i] = make_ctx<Q>(uval[i] ? u % I8<Q>::UPB : 0, uval[i] ? u / I8<Q>::UPB : 0);
  }
  using XU = std::conditional_t<F32, UnitXF<Q>, UnitX<Q>>;
  XU xu[UPT];
  if constexpr (F32) {
    // every thread loads its own units' activations (all loads issued here,
    // consumed after the ring is filled)
#pragma unroll
    for (int i = 0; i < UPT; ++i) {
      const int u = st + i * spt;
      if (uval[i]) {
        xu[i].load(p.x, p.x_mul, u / I8<Q>::UPB, u % I8<Q>::UPB);
      } else {
        xu[i].zero();
      }
    }
  } else {
    // the x loads of a row of up to 16 R blockDim.x elements in one round trip
    quantise_words<Q, b1_max_warps<Q, UPT, F32>() == 16 ? 3 : 4>(p.x, p.units, records);
  }
  // the rest of the ring: issued after x is read, so that the activation
  // loads do not queue behind a full ring of weight copies
  if (st == leader) {
    for (int i = issued; i < nst && i < ntiles; ++i, ++issued) {
      const Tile t = tile_at(p, next_issue, r1, RPS);
      issue_tile(p, p.mat_w[t.m], stages + static_cast<size_t>(i) * p.stage_stride, &full[i], t.local,
                 t.local + (t.t1 - next_issue));
      next_issue = t.t1;
    }
  }
  if constexpr (!F32) __syncthreads();  // the records are complete
  if (ntiles == 0) {  // the whole slot leaves together
    if (st == leader) gather_arrive(p, g_world, slots);
    return;
  }
  if constexpr (F32) {
#pragma unroll
    for (int i = 0; i < UPT; ++i) xu[i].finish();
    if (p.x_norm_w) {
      // the slot's threads hold every unit of x once: reduce the sum of
      // squares over the slot (the second half of the slot's reduction
      // buffer is first written after the first tile's barrier)
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < UPT; ++i) ss += xu[i].sum_squares();
      ss = warp_sum(ss);
      if (p.wps > 1) {
        float* rb = red + p.wps * RPS;
        if (lane == 0) rb[warp - slot * p.wps] = ss;
        named_barrier_sync(1 + slot, spt);
        ss = 0.f;
        for (int w = 0; w < p.wps; ++w) ss += rb[w];
      }
      const float inv = 1.0f / sqrtf(ss / static_cast<float>(p.k) + p.x_norm_eps);
#pragma unroll
      for (int i = 0; i < UPT; ++i)
        if (uval[i]) xu[i].normalise(inv, p.x_norm_w);
    }
#pragma unroll
    for (int i = 0; i < UPT; ++i) xu[i].sums();
  } else {
#pragma unroll
    for (int i = 0; i < UPT; ++i) {
      if (uval[i]) {
        xu[i].from_record(records + (st + i * spt) * RW);
      } else {
        xu[i].zero();
      }
    }
  }

  const int wis = warp - slot * p.wps;  // warp index inside the slot
  const uint32_t stages_s = smem_u32(stages);
  int64_t t0 = r0;  // consumers' cursor
  int s = 0;          // stage of tile it (it % nst, kept incrementally)
  uint32_t ph = 0u;   // its mbarrier phase parity ((it / nst) & 1)
  for (int it = 0; it < ntiles; ++it) {
    const Tile tile = tile_at(p, t0, r1, RPS);
    const int rows = static_cast<int>(tile.t1 - t0);
    float* ym = p.mat_y[tile.m] + tile.local;
    float acc[RPS];
#pragma unroll
    for (int r = 0; r < RPS; ++r) acc[r] = 0.f;
    if (wait_phase(&full[s], ph, abort)) {
      // shared address of the tile's first row: the copy keeps the source's
      // offset modulo 16 (only the low bits of the product matter)
      const uint32_t base = stages_s + static_cast<uint32_t>(s) * static_cast<uint32_t>(p.stage_stride) +
                            ((static_cast<uint32_t>(tile.local) * static_cast<uint32_t>(p.row_bytes)) & 15u);
      // A thread without a unit (its row's units do not fill the slot's last
      // warp) runs the same instructions on unit 0's bytes with zero
      // activations, and a select drops the result: no divergent branch.
      // A short tile (its row count is uniform across the slot) stops at
      // its last row; a full one has no per-row test, so the rows'
      // independent instruction streams can be interleaved.
      if (rows == RPS) {
#pragma unroll
        for (int i = 0; i < UPT; ++i) {
#pragma unroll
          for (int r = 0; r < RPS; ++r) {
            const float v = unit_dot<Q, F32>(base + static_cast<uint32_t>(r * p.row_bytes), cx[i], xu[i]);
            acc[r] += uval[i] ? v : 0.0f;
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < RPS; ++r) {
          if (r < rows) {
#pragma unroll
            for (int i = 0; i < UPT; ++i) {
              const float v = unit_dot<Q, F32>(base + static_cast<uint32_t>(r * p.row_bytes), cx[i], xu[i]);
              acc[r] += uval[i] ? v : 0.0f;
            }
          }
        }
      }
    } else if (st == 0) {
      atomicOr(p.status, kStatusFullWaitTimeout);
    }

    butterfly<RPS>(acc, lane);
    constexpr int kLanesPerValue = 32 / RPS;
    const bool refill = st == leader && it + nst < ntiles && !*abort;
    if (p.wps == 1) {
      // one warp owns the row: lane l holds row l / kLanesPerValue
      __syncwarp();  // every lane has finished reading stage s
    } else {
      float* rb = red + (it & 1) * p.wps * RPS;
      if ((lane & (kLanesPerValue - 1)) == 0) rb[wis * RPS + lane / kLanesPerValue] = acc[0];
      named_barrier_sync(1 + slot, spt);
      if (st < rows) {
        float v = 0.f;
        for (int w = 0; w < p.wps; ++w) v += rb[w * RPS + st];
        acc[0] = v;
      }
    }
    if (refill) {
      // the stage is free: every thread of the slot has passed the barrier
      const Tile nt = tile_at(p, next_issue, r1, RPS);
      fence_proxy_async_smem();
      issue_tile(p, p.mat_w[nt.m], stages + static_cast<size_t>(s) * p.stage_stride, &full[s], nt.local,
                 nt.local + (nt.t1 - next_issue));
      next_issue = nt.t1;
      ++issued;
    }
    if (p.wps == 1) {
      if ((lane & (kLanesPerValue - 1)) == 0 && lane / kLanesPerValue < rows && !*abort) {
        put_y(p, g_world, ym + lane / kLanesPerValue, acc[0]);
      }
    } else if (st < rows && !*abort) {
      put_y(p, g_world, ym + st, acc[0]);
    }
    t0 = tile.t1;
    if (++s == nst) {
      s = 0;
      ph ^= 1u;
    }
  }
  if (g_world > 1) {  // publish this slot's gathered rows
    // the leader's system fence after the slot barrier orders every thread's
    // stores of the slot before the arrival (fences are cumulative)
    if (p.wps == 1) {
      __syncwarp();
    } else {
      named_barrier_sync(1 + slot, spt);
    }
    if (st == leader) gather_arrive(p, g_world, slots);
  }

  // on an abort, copies already issued must land before the CTA exits
  if (st == leader && *abort) {
    const int first = issued > nst ? issued - nst : 0;
    int zero = 0;
    for (int i = first; i < issued; ++i) {
      if (!wait_phase(&full[i % nst], static_cast<uint32_t>(i / nst) & 1u, &zero)) {
        atomicOr(p.status, kStatusDrainTimeout);
      }
    }
  }
}

// Bytes before the stages: barriers, reduction buffers, activation records
// (integer grid only).
template <int Q, int RPS, bool F32>
__host__ __device__ constexpr int b1_smem_header(int slots, int nst, int wps, int units) {
  return (((slots * nst * 8 + 4 + 15) / 16) * 16 + ((slots * 2 * wps * RPS * 4 + 15) / 16) * 16 +
          units * (F32 ? 0 : record_words<Q>()) * 4 + 127) / 128 * 128;
}

// ---------------------------------------------------------------------------
// batch 2..BMAX, activations through L1
// ---------------------------------------------------------------------------
template <int Q, int RT, int BMAX>
__global__ void __launch_bounds__((kMaxConsumerWarps + 1) * 32, 1) gemv_xb(GemvParams p) {
  using F = Fmt<Q>;
  constexpr int E = 16 * F::NRUN;
  constexpr int V = RT * BMAX;  // values reduced per tile, index b*RT + r
  constexpr int VW = V < 32 ? V : 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const SmemLayout L = carve<V>(smem, p.nstage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncw = static_cast<int>(blockDim.x >> 5) - 1;
  const int nct = ncw * 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nstage; ++s) {
      mbar_init(&L.full[s], 1);
      mbar_init(&L.empty[s], ncw);
    }
    *L.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();

  int64_t r0, r1;
  cta_rows(p.n, r0, r1);

  if (warp == ncw) {
    if (lane == 0) produce(p, L, r0, r1, RT);
    return;
  }

  volatile int* abort = L.abort;
  int it = 0;
  for (int64_t t0 = r0; t0 < r1; t0 += RT, ++it) {
    const int s = it % p.nstage;
    const uint32_t ph = static_cast<uint32_t>(it / p.nstage) & 1u;
    const int rows = static_cast<int>((t0 + RT < r1 ? t0 + RT : r1) - t0);
    float acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0.f;
    if (wait_phase(&L.full[s], ph, abort)) {
      const uint8_t* base = L.stages + static_cast<size_t>(s) * p.stage_stride +
                            ((static_cast<uint64_t>(t0) * p.row_bytes) & 15u);
      for (int u = threadIdx.x; u < p.units; u += nct) {
        const int b = u / F::UPB, j = u % F::UPB;
        const float* xb = p.x + static_cast<int64_t>(b) * F::QK;
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          if (r < rows) {
            float wv[E];
            UnitDecode<Q>::run(base + r * p.row_bytes + b * F::TS, j, wv);
#pragma unroll
            for (int c = 0; c < BMAX; ++c) {
              if (c < p.batch) {
                float a = 0.f;
#pragma unroll
                for (int rr = 0; rr < F::NRUN; ++rr) {
                  float xr[16];
                  load_run16(xb + static_cast<int64_t>(c) * p.k + run_start<Q>(j, rr), xr);
#pragma unroll
                  for (int e = 0; e < 16; ++e) a = fmaf(wv[16 * rr + e], xr[e], a);
                }
                acc[c * RT + r] += a;
              }
            }
          }
        }
      }
    } else {
      atomicOr(p.status, kStatusFullWaitTimeout);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&L.empty[s]);

    float* red = L.red + (it & 1) * kMaxConsumerWarps * V;
    constexpr int kLanesPerValue = 32 / VW;
#pragma unroll
    for (int c0 = 0; c0 < V; c0 += 32) {
      float part[VW];
#pragma unroll
      for (int i = 0; i < VW; ++i) part[i] = acc[c0 + i];
      butterfly<VW>(part, lane);
      if ((lane & (kLanesPerValue - 1)) == 0) red[warp * V + c0 + lane / kLanesPerValue] = part[0];
    }
    named_barrier_sync(1, nct);
    if (warp == 0) {
      for (int v = lane; v < V; v += 32) {
        const int r = v % RT, c = v / RT;
        if (r < rows && c < p.batch) {
          float sum = 0.f;
          for (int w = 0; w < ncw; ++w) sum += red[w * V + v];
          if (!*abort) p.y[static_cast<int64_t>(c) * p.n + t0 + r] = sum;
        }
      }
    }
  }
}

}  // namespace frc
