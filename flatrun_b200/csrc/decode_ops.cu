// Device-resident decoder-step operators: everything a Qwen2/Llama decode
// token needs around the projections, so a whole token runs on the GPU with
// no host round trip between layers (and can be captured in one CUDA graph).
//
// They restate the reference forwarder's NumPy steps
// (src/flatrun/model/qwen2.py):
//   RMSNorm                         :365-378  x * (1 / sqrt(mean(x^2) + eps)) * w
//   q/k/v bias, RoPE (rotate-half)  :1527-1583, :398-476
//   KV append                       :1585-1595
//   GQA attention, scaled scores,
//   causal softmax, A.V             :1597-1614, :480-509
//   embedding row                   :2153-2159
// The position of the token is read from device memory (one int per
// sequence), so the same launches replay for every token.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <cstdio>

#include "../../include/frcuda.h"
#include "gemv.cuh"

namespace frc {

// Programmatic dependent launch: every kernel here waits for the previous
// kernel of the stream before touching memory, and lets the next one launch
// at once (its own wait keeps it ordered after this kernel's end), so the
// next GEMV can stream its first weight tiles while this kernel runs.
FRC_DEVICE_INLINE void pdl_enter() {
  griddep_wait();
  griddep_launch_dependents();
}

// ---------------------------------------------------------------------------
// RMSNorm of `rows` rows of n fp32 values: one CTA per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                      int n, float eps, float* __restrict__ out) {
  pdl_enter();
  const float* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  float* yr = out + static_cast<int64_t>(blockIdx.x) * n;
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
  __shared__ float red[32];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(red[0] / static_cast<float>(n) + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = (xr[i] * inv) * w[i];
}

// ---------------------------------------------------------------------------
// q/k/v bias, rotate-half RoPE at position *pos, K/V append.  qkv holds q
// (nh * hd), k (nkv * hd) and v (nkv * hd) of one token back to back; q is
// rotated in place; the rotated k and the v go to row *pos of the caches
// (layout [max_pos][nkv][hd]).  cos/sin tables are [max_pos][hd / 2].
// One thread per rotation pair (q and k) or per v element.
// ---------------------------------------------------------------------------
__global__ void rope_append_kernel(float* __restrict__ qkv, const float* __restrict__ bias, int nh, int nkv, int hd,
                                   const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                   const int* __restrict__ pos_ptr, float* __restrict__ k_cache,
                                   float* __restrict__ v_cache) {
  pdl_enter();
  const int pos = *pos_ptr;
  const int half = hd / 2;
  const int nq_pairs = nh * half, nk_pairs = nkv * half, nv = nkv * hd;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const float* c = cos_t + static_cast<int64_t>(pos) * half;
  const float* s = sin_t + static_cast<int64_t>(pos) * half;
  if (t < nq_pairs + nk_pairs) {
    const bool is_q = t < nq_pairs;
    const int u = is_q ? t : t - nq_pairs;
    const int head = u / half, i = u % half;
    const int off = (is_q ? 0 : nh * hd) + head * hd;
    float a = qkv[off + i], b = qkv[off + i + half];
    if (bias) {
      a += bias[off + i];
      b += bias[off + i + half];
    }
    const float ra = a * c[i] - b * s[i];
    const float rb = b * c[i] + a * s[i];
    if (is_q) {
      qkv[off + i] = ra;
      qkv[off + i + half] = rb;
    } else {
      float* kr = k_cache + (static_cast<int64_t>(pos) * nkv + head) * hd;
      kr[i] = ra;
      kr[i + half] = rb;
    }
  } else if (t < nq_pairs + nk_pairs + nv) {
    const int e = t - nq_pairs - nk_pairs;
    const int off = (nh + nkv) * hd + e;
    float v = qkv[off];
    if (bias) v += bias[off];
    v_cache[static_cast<int64_t>(pos) * nv + e] = v;
  }
}

// ---------------------------------------------------------------------------
// Decode attention (one query token) over positions [0, *pos] of the caches,
// split over positions ("flash decoding"): CTA (g, c) takes KV head g and
// the c-th of `splits` position ranges, with the G = nh / nkv query heads
// that read that KV head (GQA: query head h reads KV head h / G).  Head dim
// HD (64 or 128): lane l of a warp owns dimensions VEC*l.. (VEC = HD / 32),
// so every K or V row is one coalesced warp load.  Per chunk of positions:
//   scores: warp w takes positions w, w+8, ...; the lanes' partial dots of
//     the G heads are summed with one butterfly (G <= 8 values, 9 shuffles);
//   softmax: per head, the chunk's max and sum of exp(score - max);
//   A.V: warp w accumulates exp(score - max) * V over its positions, then
//     merges into its running (max, sum, acc) per head.
// The eight warps' accumulators are added at the end; the range's partial
// (max, sum, acc[G][128]) goes to `part` for attn_combine.
// ---------------------------------------------------------------------------
constexpr int kAttnThreads = 256;
constexpr int kAttnMaxHd = 128;
constexpr int kAttnMaxG = 8;
constexpr int kAttnChunk = 256;  // positions per pass of a range

// VEC consecutive floats at p (16- or 8-byte aligned).
template <int VEC>
FRC_DEVICE_INLINE void load_vec(const float* p, float (&v)[VEC]) {
  if constexpr (VEC == 4) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
    static_assert(VEC == 2, "head_dim 64 or 128");
    const float2 t = *reinterpret_cast<const float2*>(p);
    v[0] = t.x; v[1] = t.y;
  }
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_partial_kernel(
    const float* __restrict__ q, const float* __restrict__ k_cache, const float* __restrict__ v_cache,
    const int* __restrict__ pos_ptr, int nh, int nkv, float scale, int splits, float* __restrict__ part) {
  pdl_enter();
  constexpr int MG = kAttnMaxG, NW = kAttnThreads / 32, VEC = HD / 32;
  const int g = blockIdx.x, c = blockIdx.y;
  const int G = nh / nkv;
  const int total = *pos_ptr + 1;
  const int per = (total + splits - 1) / splits;
  const int t0 = c * per, t1 = min(total, t0 + per);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ __align__(16) float sc[kAttnChunk][MG];  // scores, then exp(score - max)
  __shared__ float cmax[MG], csum[MG];
  __shared__ __align__(16) float wacc[NW][MG][HD];

  float qv[MG][VEC];
#pragma unroll
  for (int h = 0; h < MG; ++h) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) qv[h][e] = 0.f;
    if (h < G) load_vec<VEC>(q + (g * G + h) * HD + VEC * lane, qv[h]);
  }
  float m_run[MG], l_run[MG], acc[MG][VEC];
#pragma unroll
  for (int h = 0; h < MG; ++h) {
    m_run[h] = -FLT_MAX;
    l_run[h] = 0.f;
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[h][e] = 0.f;
  }
  const int64_t row_stride = static_cast<int64_t>(nkv) * HD;
  const float* kb = k_cache + static_cast<int64_t>(g) * HD + VEC * lane;
  const float* vb = v_cache + static_cast<int64_t>(g) * HD + VEC * lane;
  for (int base = t0; base < t1; base += kAttnChunk) {
    const int n_t = min(kAttnChunk, t1 - base);
    // scores: each warp takes eight positions per pass so that eight row
    // loads are in flight at once
    for (int t = warp; t < n_t; t += 8 * NW) {
      float kr[8][VEC];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) kr[u][e] = 0.f;
        if (t + u * NW < n_t) load_vec<VEC>(kb + (base + t + u * NW) * row_stride, kr[u]);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float sv[MG];
#pragma unroll
        for (int h = 0; h < MG; ++h) {
          sv[h] = 0.f;
#pragma unroll
          for (int e = 0; e < VEC; ++e) sv[h] = fmaf(qv[h][e], kr[u][e], sv[h]);
        }
        butterfly<MG>(sv, lane);
        // lane l now holds head l / 4's total
        if ((lane & 3) == 0 && (lane >> 2) < G && t + u * NW < n_t) sc[t + u * NW][lane >> 2] = sv[0] * scale;
      }
    }
    __syncthreads();
    // per head: the chunk's max, then exp(score - max) and their sum
    for (int h = warp; h < G; h += NW) {
      float m = -FLT_MAX;
      for (int t = lane; t < n_t; t += 32) m = fmaxf(m, sc[t][h]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float l = 0.f;
      for (int t = lane; t < n_t; t += 32) {
        const float e = expf(sc[t][h] - m);
        sc[t][h] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        cmax[h] = m;
        csum[h] = l;
      }
    }
    __syncthreads();
    // A.V over this warp's positions of the chunk
    float a[MG][VEC];
#pragma unroll
    for (int h = 0; h < MG; ++h)
#pragma unroll
      for (int e = 0; e < VEC; ++e) a[h][e] = 0.f;
    for (int t = warp; t < n_t; t += 8 * NW) {
      float vr[8][VEC];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) vr[u][e] = 0.f;
        if (t + u * NW < n_t) load_vec<VEC>(vb + (base + t + u * NW) * row_stride, vr[u]);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (t + u * NW < n_t) {
          const float4 p0 = *reinterpret_cast<const float4*>(&sc[t + u * NW][0]);
          const float4 p1 = *reinterpret_cast<const float4*>(&sc[t + u * NW][4]);
          const float pw[MG] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
          for (int h = 0; h < MG; ++h)
#pragma unroll
            for (int e = 0; e < VEC; ++e) a[h][e] = fmaf(pw[h], vr[u][e], a[h][e]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < MG; ++h) {
      if (h < G) {
        const float m_new = fmaxf(m_run[h], cmax[h]);
        const float e_old = expf(m_run[h] - m_new), e_blk = expf(cmax[h] - m_new);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[h][e] = acc[h][e] * e_old + a[h][e] * e_blk;
        l_run[h] = l_run[h] * e_old + csum[h] * e_blk;
        m_run[h] = m_new;
      }
    }
    __syncthreads();  // sc and cmax are rewritten by the next chunk
  }
  // add the warps' accumulators; partial layout per (head, split):
  // [max, sum, acc[HD]]
#pragma unroll
  for (int h = 0; h < MG; ++h)
#pragma unroll
    for (int e = 0; e < VEC; ++e) wacc[warp][h][VEC * lane + e] = acc[h][e];
  __syncthreads();
  for (int d = threadIdx.x; d < HD; d += kAttnThreads) {
    for (int h = 0; h < G; ++h) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) v += wacc[w][h][d];
      float* pr = part + (static_cast<int64_t>(g * G + h) * splits + c) * (HD + 2);
      if (d == 0) {
        pr[0] = m_run[h];
        pr[1] = l_run[h];
      }
      pr[2 + d] = v;
    }
  }
}

// Merge the splits of every head: out[h][d] = sum_c acc_c e^(m_c - M) /
// sum_c l_c e^(m_c - M).  One CTA per head (one thread per d); the splits'
// (max, sum) pairs are read in parallel first.
constexpr int kAttnMaxSplits = 1024;

constexpr int kCombineGroups = 8;  // threads per output element: split groups

__global__ void __launch_bounds__(kAttnMaxHd * kCombineGroups) attn_combine_kernel(
    const float* __restrict__ part, int hd, int splits, float* __restrict__ out) {
  pdl_enter();
  // blockDim = (hd, kCombineGroups): thread (d, j) sums the splits c = j mod G
  const int h = blockIdx.x, d = threadIdx.x, j = threadIdx.y;
  const int tid = j * blockDim.x + d, nthreads = blockDim.x * blockDim.y;
  const float* ph = part + static_cast<int64_t>(h) * splits * (hd + 2);
  __shared__ float em[kAttnMaxSplits];
  __shared__ float red[32];
  __shared__ float sums[kCombineGroups][kAttnMaxHd];
  __shared__ float bcast[2];
  float m = -FLT_MAX;
  for (int c = tid; c < splits; c += nthreads) m = fmaxf(m, ph[c * (hd + 2)]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) red[tid >> 5] = m;
  __syncthreads();
  if (tid == 0) {
    float M = red[0];
    for (int w = 1; w < nthreads / 32; ++w) M = fmaxf(M, red[w]);
    bcast[0] = M;
  }
  __syncthreads();
  const float M = bcast[0];
  float L = 0.f;
  for (int c = tid; c < splits; c += nthreads) {
    const float* pc = ph + c * (hd + 2);
    const float e = pc[1] == 0.f ? 0.f : expf(pc[0] - M);  // an empty range contributes nothing
    em[c] = e;
    L = fmaf(pc[1], e, L);
  }
  L = warp_sum(L);
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = L;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < nthreads / 32; ++w) t += red[w];
    bcast[1] = t;
  }
  float A = 0.f;
#pragma unroll 4
  for (int c = j; c < splits; c += kCombineGroups) A = fmaf(ph[c * (hd + 2) + 2 + d], em[c], A);
  sums[j][d] = A;
  __syncthreads();
  if (j == 0) {
    float t = 0.f;
#pragma unroll
    for (int g = 0; g < kCombineGroups; ++g) t += sums[g][d];
    out[h * hd + d] = t / bcast[1];
  }
}

// ---------------------------------------------------------------------------
// Index of the largest of n values (the lowest index among equal maxima, as
// np.argmax).  Every CTA reduces a slice into ws (value, index); the last
// CTA to finish (ticket in ws) reduces the slices and resets the ticket, so
// the kernel replays in a graph.
// ---------------------------------------------------------------------------
FRC_DEVICE_INLINE void argmax_merge(float& best, int64_t& bi, float ov, int64_t oi) {
  if (ov > best || (ov == best && oi < bi)) {
    best = ov;
    bi = oi;
  }
}

FRC_DEVICE_INLINE void argmax_block(float& best, int64_t& bi) {
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    best = threadIdx.x < nw ? sv[threadIdx.x] : -FLT_MAX;
    bi = threadIdx.x < nw ? si[threadIdx.x] : INT64_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
  }
}

constexpr int kArgmaxThreads = 256;

__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ x, int64_t n,
                                                               int* __restrict__ out, int64_t* __restrict__ ws) {
  pdl_enter();
  // ws: [0] ticket, [1 + 2b] value bits, [2 + 2b] index of CTA b
  const int64_t per = (n + gridDim.x - 1) / gridDim.x;
  const int64_t i0 = blockIdx.x * per, i1 = min(n, i0 + per);
  float best = -FLT_MAX;
  int64_t bi = INT64_MAX;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) argmax_merge(best, bi, x[i], i);
  argmax_block(best, bi);
  __shared__ bool last;
  if (threadIdx.x == 0) {
    ws[1 + 2 * blockIdx.x] = __float_as_int(best);
    ws[2 + 2 * blockIdx.x] = bi;
    __threadfence();
    last = atomicAdd(reinterpret_cast<unsigned long long*>(ws), 1ull) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  best = -FLT_MAX;
  bi = INT64_MAX;
  for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += blockDim.x) {
    const volatile int64_t* w = ws;
    argmax_merge(best, bi, __int_as_float(static_cast<int>(w[1 + 2 * b])), w[2 + 2 * b]);
  }
  argmax_block(best, bi);
  if (threadIdx.x == 0) {
    *out = static_cast<int>(bi);
    ws[0] = 0;
  }
}

// ---------------------------------------------------------------------------
// Embedding row *tok of a (vocab, n) table into out: fp32 rows copied, GGUF
// rows dequantised bit-exactly (dequant_elem, the reference NumPy decoders).
// ---------------------------------------------------------------------------
__global__ void embed_f32_kernel(const float* __restrict__ table, int n, const int* __restrict__ tok,
                                 float* __restrict__ out) {
  pdl_enter();
  const float* row = table + static_cast<int64_t>(*tok) * n;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = row[i];
}

template <int Q>
__global__ void embed_q_kernel(const uint8_t* __restrict__ table, int n, const int* __restrict__ tok,
                               float* __restrict__ out) {
  pdl_enter();
  using F = Fmt<Q>;
  const uint8_t* row = table + static_cast<int64_t>(*tok) * (n / F::QK) * F::TS;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = dequant_elem<Q>(row + (i / F::QK) * F::TS, i % F::QK);
}

// Increment the device position (one thread): the last launch of a token.
__global__ void pos_advance_kernel(int* pos) {
  pdl_enter();
  *pos += 1;
}

// Launch with the programmatic-stream-serialization attribute.
template <typename... P, typename... A>
cudaError_t launch_dep(void (*kernel)(P...), dim3 grid, dim3 block, cudaStream_t st, A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<P>(args)...);
}

}  // namespace frc

namespace {

thread_local char g_decode_err[256];

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return FRC_OK;
  snprintf(g_decode_err, sizeof g_decode_err, "%s: %s", what, cudaGetErrorString(e));
  return FRC_ERR_CUDA;
}

}  // namespace

// Defined in frcuda_api.cu: records a message for frc_last_error.
extern "C" int frc__fail(int code, const char* msg);

#define FRC_DECODE_CHECK(cond, msg) \
  do {                              \
    if (!(cond)) return frc__fail(FRC_ERR_INVALID, msg); \
  } while (0)

#define FRC_DECODE_LAUNCHED(what)                     \
  do {                                                \
    const int _rc = launch_status(what);              \
    if (_rc) return frc__fail(_rc, g_decode_err);     \
    return FRC_OK;                                    \
  } while (0)

extern "C" {

int frc_rmsnorm(const float* x, const float* w, int64_t rows, int64_t n, float eps, float* out, void* stream) {
  FRC_DECODE_CHECK(rows >= 0 && n > 0 && n <= (int64_t(1) << 30), "frc_rmsnorm: bad shape");
  FRC_DECODE_CHECK(x && w && out, "frc_rmsnorm: null pointer");
  if (rows == 0) return FRC_OK;
  frc::launch_dep(frc::rmsnorm_kernel, dim3(static_cast<unsigned>(rows)), dim3(1024), static_cast<cudaStream_t>(stream),
                  x, w, static_cast<int>(n), eps, out);
  FRC_DECODE_LAUNCHED("rmsnorm launch");
}

int frc_rope_append(float* qkv, const float* bias, int nh, int nkv, int hd, const float* cos_table,
                    const float* sin_table, const int* pos_dev, float* k_cache, float* v_cache, void* stream) {
  FRC_DECODE_CHECK(nh > 0 && nkv > 0 && nh % nkv == 0 && hd > 0 && hd % 2 == 0, "frc_rope_append: bad heads");
  FRC_DECODE_CHECK(qkv && cos_table && sin_table && pos_dev && k_cache && v_cache, "frc_rope_append: null pointer");
  const int threads = nh * hd / 2 + nkv * hd / 2 + nkv * hd;
  frc::launch_dep(frc::rope_append_kernel, dim3((threads + 255) / 256), dim3(256), static_cast<cudaStream_t>(stream),
                  qkv, bias, nh, nkv, hd, cos_table, sin_table, pos_dev, k_cache, v_cache);
  FRC_DECODE_LAUNCHED("rope_append launch");
}

int frc_attention_decode(const float* q, const float* k_cache, const float* v_cache, const int* pos_dev, int nh,
                         int nkv, int hd, float scale, int splits, float* part, float* out, void* stream) {
  FRC_DECODE_CHECK(nh > 0 && nkv > 0 && nh % nkv == 0 && nh / nkv <= frc::kAttnMaxG,
                   "frc_attention_decode: needs nh a multiple of nkv and at most 8 query heads per KV head");
  FRC_DECODE_CHECK(hd == 64 || hd == 128, "frc_attention_decode: head_dim must be 64 or 128");
  FRC_DECODE_CHECK(splits >= 1 && splits <= frc::kAttnMaxSplits, "frc_attention_decode: splits must be 1..1024");
  FRC_DECODE_CHECK(q && k_cache && v_cache && pos_dev && part && out, "frc_attention_decode: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (hd == 128)
    frc::launch_dep(frc::attn_partial_kernel<128>, dim3(nkv, splits), dim3(frc::kAttnThreads), st, q, k_cache, v_cache,
                    pos_dev, nh, nkv, scale, splits, part);
  else
    frc::launch_dep(frc::attn_partial_kernel<64>, dim3(nkv, splits), dim3(frc::kAttnThreads), st, q, k_cache, v_cache,
                    pos_dev, nh, nkv, scale, splits, part);
  int rc = launch_status("attention launch");
  if (rc) return frc__fail(rc, g_decode_err);
  frc::launch_dep(frc::attn_combine_kernel, dim3(nh), dim3(hd, frc::kCombineGroups), st, part, hd, splits, out);
  FRC_DECODE_LAUNCHED("attention combine launch");
}

int frc_attention_workspace(int nh, int hd, int splits, size_t* floats) {
  FRC_DECODE_CHECK(floats && nh > 0 && hd > 0 && splits > 0, "frc_attention_workspace: bad arguments");
  *floats = static_cast<size_t>(nh) * splits * (hd + 2);
  return FRC_OK;
}

int frc_argmax_workspace(int64_t n, size_t* bytes) {
  FRC_DECODE_CHECK(bytes && n > 0, "frc_argmax_workspace: bad arguments");
  *bytes = 8 * (1 + 2 * 148 * 2);  // ticket + (value, index) per CTA, up to 296 CTAs
  return FRC_OK;
}

int frc_argmax(const float* x, int64_t n, int* out_dev, void* workspace, void* stream) {
  FRC_DECODE_CHECK(x && out_dev && workspace && n > 0, "frc_argmax: null pointer or empty input");
  int64_t grid = (n + 4 * frc::kArgmaxThreads - 1) / (4 * frc::kArgmaxThreads);
  if (grid > 296) grid = 296;
  frc::launch_dep(frc::argmax_kernel, dim3(static_cast<unsigned>(grid)), dim3(frc::kArgmaxThreads),
                  static_cast<cudaStream_t>(stream), x, n, out_dev, static_cast<int64_t*>(workspace));
  FRC_DECODE_LAUNCHED("argmax launch");
}

int frc_embed_row(int quant, const void* table, int64_t n, const int* tok_dev, float* out, void* stream) {
  FRC_DECODE_CHECK(table && tok_dev && out && n > 0, "frc_embed_row: null pointer or empty row");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256 < 64 ? (n + 255) / 256 : 64);
  const int in = static_cast<int>(n);
  switch (quant) {
    case 0:
      frc::launch_dep(frc::embed_f32_kernel, dim3(blocks), dim3(256), st, static_cast<const float*>(table), in, tok_dev,
                      out);
      break;
    case FRC_Q8_0:
    case FRC_Q4_K:
    case FRC_Q5_K:
    case FRC_Q6_K:
    case FRC_Q1_0: {
      const int qk = quant == FRC_Q8_0 ? 32 : (quant == FRC_Q1_0 ? 128 : 256);
      FRC_DECODE_CHECK(n % qk == 0, "frc_embed_row: row length must be a multiple of the block size");
      const uint8_t* t = static_cast<const uint8_t*>(table);
      if (quant == FRC_Q8_0) frc::launch_dep(frc::embed_q_kernel<frc::kQ8_0>, dim3(blocks), dim3(256), st, t, in, tok_dev, out);
      if (quant == FRC_Q4_K) frc::launch_dep(frc::embed_q_kernel<frc::kQ4_K>, dim3(blocks), dim3(256), st, t, in, tok_dev, out);
      if (quant == FRC_Q5_K) frc::launch_dep(frc::embed_q_kernel<frc::kQ5_K>, dim3(blocks), dim3(256), st, t, in, tok_dev, out);
      if (quant == FRC_Q6_K) frc::launch_dep(frc::embed_q_kernel<frc::kQ6_K>, dim3(blocks), dim3(256), st, t, in, tok_dev, out);
      if (quant == FRC_Q1_0) frc::launch_dep(frc::embed_q_kernel<frc::kQ1_0>, dim3(blocks), dim3(256), st, t, in, tok_dev, out);
      break;
    }
    default: return frc__fail(FRC_ERR_INVALID, "frc_embed_row: quant must be 0 (fp32) or a supported GGUF type");
  }
  FRC_DECODE_LAUNCHED("embed launch");
}

int frc_pos_advance(int* pos_dev, void* stream) {
  FRC_DECODE_CHECK(pos_dev, "frc_pos_advance: null pointer");
  frc::launch_dep(frc::pos_advance_kernel, dim3(1), dim3(1), static_cast<cudaStream_t>(stream), pos_dev);
  FRC_DECODE_LAUNCHED("pos_advance launch");
}

}  // extern "C"
