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
#include "formats.cuh"

namespace frc {

// ---------------------------------------------------------------------------
// RMSNorm of `rows` rows of n fp32 values: one CTA per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                      int n, float eps, float* __restrict__ out) {
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
// that read that KV head (GQA: query head h reads KV head h / G).
//   phase 1: thread t scores position t of the range for every query head;
//   phase 2: per head, the range's max and sum of exp(score - max);
//   phase 3: thread d accumulates sum_t exp(score - max) * V[t][d] per head.
// Partials (max, sum, acc[G][hd]) go to `part`; attn_combine merges them.
// hd <= 128, G <= 16, blockDim.x = 128.
// ---------------------------------------------------------------------------
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxHd = 128;
constexpr int kAttnMaxG = 16;
constexpr int kAttnChunk = 128;  // positions scored per pass of a range

__global__ void __launch_bounds__(kAttnThreads) attn_partial_kernel(
    const float* __restrict__ q, const float* __restrict__ k_cache, const float* __restrict__ v_cache,
    const int* __restrict__ pos_ptr, int nh, int nkv, int hd, float scale, int splits, float* __restrict__ part) {
  const int g = blockIdx.x, c = blockIdx.y;
  const int G = nh / nkv;
  const int total = *pos_ptr + 1;
  const int per = (total + splits - 1) / splits;
  const int t0 = c * per, t1 = min(total, t0 + per);
  __shared__ float qs[kAttnMaxG][kAttnMaxHd];
  __shared__ float sc[kAttnMaxG][kAttnChunk];
  __shared__ float red[kAttnMaxG][2];
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) qs[i / hd][i % hd] = q[(g * G + i / hd) * hd + i % hd];
  float m_run[kAttnMaxG], l_run[kAttnMaxG], acc[kAttnMaxG];
#pragma unroll
  for (int h = 0; h < kAttnMaxG; ++h) {
    m_run[h] = -FLT_MAX;
    l_run[h] = 0.f;
    acc[h] = 0.f;
  }
  __syncthreads();
  const int d = threadIdx.x;
  for (int base = t0; base < t1; base += kAttnChunk) {
    const int n_t = min(kAttnChunk, t1 - base);
    // phase 1: scores of position base + tid for every head
    if (threadIdx.x < n_t) {
      const float4* kr = reinterpret_cast<const float4*>(k_cache + (static_cast<int64_t>(base + threadIdx.x) * nkv + g) * hd);
      float s[kAttnMaxG];
#pragma unroll
      for (int h = 0; h < kAttnMaxG; ++h) s[h] = 0.f;
      for (int i = 0; i < hd / 4; ++i) {
        const float4 kv = kr[i];
#pragma unroll
        for (int h = 0; h < kAttnMaxG; ++h) {
          if (h < G) {
            s[h] = fmaf(qs[h][4 * i], kv.x, s[h]);
            s[h] = fmaf(qs[h][4 * i + 1], kv.y, s[h]);
            s[h] = fmaf(qs[h][4 * i + 2], kv.z, s[h]);
            s[h] = fmaf(qs[h][4 * i + 3], kv.w, s[h]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < kAttnMaxG; ++h)
        if (h < G) sc[h][threadIdx.x] = s[h] * scale;
    }
    __syncthreads();
    // phase 2: the chunk's max per head (warp h % 4 reduces head h), the
    // running max and sum rescaled to it
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int h = warp; h < G; h += kAttnThreads / 32) {
      float m = -FLT_MAX;
      for (int t = lane; t < n_t; t += 32) m = fmaxf(m, sc[h][t]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float l = 0.f;
      for (int t = lane; t < n_t; t += 32) {
        const float e = expf(sc[h][t] - m);
        sc[h][t] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        red[h][0] = m;
        red[h][1] = l;
      }
    }
    __syncthreads();
    // phase 3: merge into the running (max, sum, acc) of every head
    if (d < hd) {
      for (int h = 0; h < G; ++h) {
        const float m_new = fmaxf(m_run[h], red[h][0]);
        const float a_old = expf(m_run[h] - m_new), a_blk = expf(red[h][0] - m_new);
        float s = 0.f;
        for (int t = 0; t < n_t; ++t)
          s = fmaf(sc[h][t], v_cache[(static_cast<int64_t>(base + t) * nkv + g) * hd + d], s);
        acc[h] = acc[h] * a_old + s * a_blk;
        l_run[h] = l_run[h] * a_old + red[h][1] * a_blk;
        m_run[h] = m_new;
      }
    }
    __syncthreads();
  }
  // partial layout per (head, split): [max, sum, acc[hd]]
  if (d < hd) {
    for (int h = 0; h < G; ++h) {
      float* pr = part + (static_cast<int64_t>(g * G + h) * splits + c) * (hd + 2);
      if (d == 0) {
        pr[0] = m_run[h];
        pr[1] = l_run[h];
      }
      pr[2 + d] = acc[h];
    }
  }
}

// Merge the splits of every head: out[h][d] = sum_c acc_c e^(m_c - M) /
// sum_c l_c e^(m_c - M).  One CTA per head, one thread per d.
__global__ void attn_combine_kernel(const float* __restrict__ part, int hd, int splits, float* __restrict__ out) {
  const int h = blockIdx.x, d = threadIdx.x;
  if (d >= hd) return;
  const float* ph = part + static_cast<int64_t>(h) * splits * (hd + 2);
  float M = -FLT_MAX;
  for (int c = 0; c < splits; ++c) M = fmaxf(M, ph[c * (hd + 2)]);
  float L = 0.f, A = 0.f;
  for (int c = 0; c < splits; ++c) {
    const float* pc = ph + c * (hd + 2);
    if (pc[1] == 0.f) continue;  // an empty range
    const float e = expf(pc[0] - M);
    L = fmaf(pc[1], e, L);
    A = fmaf(pc[2 + d], e, A);
  }
  out[h * hd + d] = A / L;
}

// ---------------------------------------------------------------------------
// Index of the largest of n values (the lowest index among equal maxima, as
// np.argmax): one CTA.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ x, int64_t n, int* __restrict__ out) {
  float best = -FLT_MAX;
  int64_t bi = 0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    if (v > best) {
      best = v;
      bi = i;
    }
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
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
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) *out = static_cast<int>(bi);
  }
}

// ---------------------------------------------------------------------------
// Embedding row *tok of a (vocab, n) table into out: fp32 rows copied, GGUF
// rows dequantised bit-exactly (dequant_elem, the reference NumPy decoders).
// ---------------------------------------------------------------------------
__global__ void embed_f32_kernel(const float* __restrict__ table, int n, const int* __restrict__ tok,
                                 float* __restrict__ out) {
  const float* row = table + static_cast<int64_t>(*tok) * n;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = row[i];
}

template <int Q>
__global__ void embed_q_kernel(const uint8_t* __restrict__ table, int n, const int* __restrict__ tok,
                               float* __restrict__ out) {
  using F = Fmt<Q>;
  const uint8_t* row = table + static_cast<int64_t>(*tok) * (n / F::QK) * F::TS;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = dequant_elem<Q>(row + (i / F::QK) * F::TS, i % F::QK);
}

// Increment the device position (one thread): the last launch of a token.
__global__ void pos_advance_kernel(int* pos) { *pos += 1; }

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
  frc::rmsnorm_kernel<<<static_cast<unsigned>(rows), 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      x, w, static_cast<int>(n), eps, out);
  FRC_DECODE_LAUNCHED("rmsnorm launch");
}

int frc_rope_append(float* qkv, const float* bias, int nh, int nkv, int hd, const float* cos_table,
                    const float* sin_table, const int* pos_dev, float* k_cache, float* v_cache, void* stream) {
  FRC_DECODE_CHECK(nh > 0 && nkv > 0 && nh % nkv == 0 && hd > 0 && hd % 2 == 0, "frc_rope_append: bad heads");
  FRC_DECODE_CHECK(qkv && cos_table && sin_table && pos_dev && k_cache && v_cache, "frc_rope_append: null pointer");
  const int threads = nh * hd / 2 + nkv * hd / 2 + nkv * hd;
  frc::rope_append_kernel<<<(threads + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      qkv, bias, nh, nkv, hd, cos_table, sin_table, pos_dev, k_cache, v_cache);
  FRC_DECODE_LAUNCHED("rope_append launch");
}

int frc_attention_decode(const float* q, const float* k_cache, const float* v_cache, const int* pos_dev, int nh,
                         int nkv, int hd, float scale, int splits, float* part, float* out, void* stream) {
  FRC_DECODE_CHECK(nh > 0 && nkv > 0 && nh % nkv == 0 && nh / nkv <= frc::kAttnMaxG, "frc_attention_decode: bad heads");
  FRC_DECODE_CHECK(hd > 0 && hd <= frc::kAttnMaxHd && hd % 4 == 0, "frc_attention_decode: head_dim must be 4..128, a multiple of 4");
  FRC_DECODE_CHECK(splits >= 1 && splits <= 1024, "frc_attention_decode: splits must be 1..1024");
  FRC_DECODE_CHECK(q && k_cache && v_cache && pos_dev && part && out, "frc_attention_decode: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  frc::attn_partial_kernel<<<dim3(nkv, splits), frc::kAttnThreads, 0, st>>>(q, k_cache, v_cache, pos_dev, nh, nkv,
                                                                            hd, scale, splits, part);
  int rc = launch_status("attention launch");
  if (rc) return frc__fail(rc, g_decode_err);
  frc::attn_combine_kernel<<<nh, hd, 0, st>>>(part, hd, splits, out);
  FRC_DECODE_LAUNCHED("attention combine launch");
}

int frc_attention_workspace(int nh, int hd, int splits, size_t* floats) {
  FRC_DECODE_CHECK(floats && nh > 0 && hd > 0 && splits > 0, "frc_attention_workspace: bad arguments");
  *floats = static_cast<size_t>(nh) * splits * (hd + 2);
  return FRC_OK;
}

int frc_argmax(const float* x, int64_t n, int* out_dev, void* stream) {
  FRC_DECODE_CHECK(x && out_dev && n > 0, "frc_argmax: null pointer or empty input");
  frc::argmax_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, n, out_dev);
  FRC_DECODE_LAUNCHED("argmax launch");
}

int frc_embed_row(int quant, const void* table, int64_t n, const int* tok_dev, float* out, void* stream) {
  FRC_DECODE_CHECK(table && tok_dev && out && n > 0, "frc_embed_row: null pointer or empty row");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256 < 64 ? (n + 255) / 256 : 64);
  const int in = static_cast<int>(n);
  switch (quant) {
    case 0: frc::embed_f32_kernel<<<blocks, 256, 0, st>>>(static_cast<const float*>(table), in, tok_dev, out); break;
    case FRC_Q8_0:
    case FRC_Q4_K:
    case FRC_Q5_K:
    case FRC_Q6_K:
    case FRC_Q1_0: {
      const int qk = quant == FRC_Q8_0 ? 32 : (quant == FRC_Q1_0 ? 128 : 256);
      FRC_DECODE_CHECK(n % qk == 0, "frc_embed_row: row length must be a multiple of the block size");
      const uint8_t* t = static_cast<const uint8_t*>(table);
      if (quant == FRC_Q8_0) frc::embed_q_kernel<frc::kQ8_0><<<blocks, 256, 0, st>>>(t, in, tok_dev, out);
      if (quant == FRC_Q4_K) frc::embed_q_kernel<frc::kQ4_K><<<blocks, 256, 0, st>>>(t, in, tok_dev, out);
      if (quant == FRC_Q5_K) frc::embed_q_kernel<frc::kQ5_K><<<blocks, 256, 0, st>>>(t, in, tok_dev, out);
      if (quant == FRC_Q6_K) frc::embed_q_kernel<frc::kQ6_K><<<blocks, 256, 0, st>>>(t, in, tok_dev, out);
      if (quant == FRC_Q1_0) frc::embed_q_kernel<frc::kQ1_0><<<blocks, 256, 0, st>>>(t, in, tok_dev, out);
      break;
    }
    default: return frc__fail(FRC_ERR_INVALID, "frc_embed_row: quant must be 0 (fp32) or a supported GGUF type");
  }
  FRC_DECODE_LAUNCHED("embed launch");
}

int frc_pos_advance(int* pos_dev, void* stream) {
  FRC_DECODE_CHECK(pos_dev, "frc_pos_advance: null pointer");
  frc::pos_advance_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(pos_dev);
  FRC_DECODE_LAUNCHED("pos_advance launch");
}

}  // extern "C"
