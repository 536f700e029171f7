// C ABI of libfrcuda.so (declared in include/frcuda.h).
//
// Argument checks mirror the reference pybind11 boundary
// (src/flatrun_native/_C.cpp:99-138, :154-283, :285-433): k must be a
// multiple of the block size, the weight must have exactly n*(k/QK)*TS bytes,
// x must have k columns.  They run before any CUDA call, so they behave the
// same on a machine without a GPU.  No exception crosses the ABI: every entry
// point returns a status and leaves a message for frc_last_error.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/frcuda.h"
#include "launch.cuh"

namespace frc {
extern template cudaError_t launch_gemv<kQ8_0>(const GemvRequest&);
extern template cudaError_t launch_gemv<kQ4_K>(const GemvRequest&);
extern template cudaError_t launch_gemv<kQ5_K>(const GemvRequest&);
extern template cudaError_t launch_gemv<kQ6_K>(const GemvRequest&);
extern template cudaError_t launch_gemv<kQ1_0>(const GemvRequest&);
extern template cudaError_t launch_dequant<kQ8_0>(const DequantRequest&);
extern template cudaError_t launch_dequant<kQ4_K>(const DequantRequest&);
extern template cudaError_t launch_dequant<kQ5_K>(const DequantRequest&);
extern template cudaError_t launch_dequant<kQ6_K>(const DequantRequest&);
extern template cudaError_t launch_dequant<kQ1_0>(const DequantRequest&);
extern template cudaError_t launch_gemm_tc<kQ8_0>(const GemvRequest&);
extern template cudaError_t launch_gemm_tc<kQ4_K>(const GemvRequest&);
extern template cudaError_t launch_gemm_tc<kQ5_K>(const GemvRequest&);
extern template cudaError_t launch_gemm_tc<kQ6_K>(const GemvRequest&);
extern template cudaError_t launch_gemm_tc<kQ1_0>(const GemvRequest&);
}  // namespace frc

struct frc_gather {
  int world = 0, rank = 0, device = 0;
  float* shard_dst[frc::kMaxGatherRanks] = {};   // rank r's gathered buffer at this rank's shard
  uint32_t* flags[frc::kMaxGatherRanks] = {};    // rank r's flag array (one word per rank)
  uint32_t* counters = nullptr;                  // [0] slots finished, [1] epoch (this device)
};

struct frc_weight {
  int device;
  int quant;
  int64_t n, k;
  size_t nbytes;
  uint8_t* dev;
};

namespace {

constexpr int kMaxGemvBatch = 16;

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? FRC_ERR_NOMEM : FRC_ERR_CUDA, "%s: %s", what,
              cudaGetErrorString(e));
}

#define FRC_CUDA(call, what)                    \
  do {                                          \
    cudaError_t _e = (call);                    \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

bool geometry(int q, int* qk, int* ts) {
  switch (q) {
    case FRC_Q8_0: *qk = 32; *ts = 34; return true;
    case FRC_Q4_K: *qk = 256; *ts = 144; return true;
    case FRC_Q5_K: *qk = 256; *ts = 176; return true;
    case FRC_Q6_K: *qk = 256; *ts = 210; return true;
    case FRC_Q1_0: *qk = 128; *ts = 18; return true;
    default: return false;
  }
}

const char* quant_name(int q) {
  switch (q) {
    case FRC_Q8_0: return "Q8_0";
    case FRC_Q4_K: return "Q4_K";
    case FRC_Q5_K: return "Q5_K";
    case FRC_Q6_K: return "Q6_K";
    case FRC_Q1_0: return "Q1_0";
    default: return "?";
  }
}

// Checks shared by every matmul entry point; returns FRC_OK or an error.
int check_matmul(int quant, size_t w_bytes, int64_t n, int64_t k, int64_t seq) {
  int qk, ts;
  if (!geometry(quant, &qk, &ts)) return fail(FRC_ERR_INVALID, "unsupported quant id %d", quant);
  const char* q = quant_name(quant);
  if (n < 0 || k < 0) return fail(FRC_ERR_INVALID, "%s matmul: negative shape (n=%lld, k=%lld)", q, (long long)n, (long long)k);
  if (k % qk != 0) return fail(FRC_ERR_INVALID, "%s matmul: in_features must be a multiple of %d", q, qk);
  if (k > (int64_t(1) << 30)) return fail(FRC_ERR_INVALID, "%s matmul: k=%lld too large", q, (long long)k);
  if (seq < 1) return fail(FRC_ERR_INVALID, "%s matmul: batch/seq must be >= 1 (got %lld)", q, (long long)seq);
  const unsigned long long want = (unsigned long long)n * (unsigned long long)(k / qk) * (unsigned long long)ts;
  if (w_bytes != want)
    return fail(FRC_ERR_INVALID, "%s matmul: weight byte size mismatch: expected %llu bytes, got %llu", q, want,
                (unsigned long long)w_bytes);
  return FRC_OK;
}

struct DeviceState {
  int device = 0;
  int sms = 0;
  uint32_t* status = nullptr;       // device status word
  uint32_t* status_host = nullptr;  // pinned readback
  cudaStream_t stream = nullptr;    // stream of the host-buffer entry points
  std::mutex mu;                    // serialises host-buffer calls on this device
  uint8_t* scratch_w = nullptr;
  size_t cap_w = 0;
  float* scratch_x = nullptr;
  size_t cap_x = 0;
  float* scratch_y = nullptr;
  size_t cap_y = 0;
  // pinned staging of small host-buffer calls: x is copied in, y out through
  // it, so both transfers are asynchronous DMA (a pageable transfer is staged
  // by the driver through its own buffer, one synchronous copy per call)
  uint8_t* pinned = nullptr;
  size_t cap_pinned = 0;
  // device result of a host-buffer matmul: a kHostOutHead-byte head whose
  // first word is the call's own status word (zero between calls), then y;
  // one device-to-host copy returns both
  uint8_t* host_out = nullptr;
  size_t cap_host_out = 0;
  // activation records of the batched tensor-core kernel: grown on demand and
  // never freed while the process runs, so work already queued (or captured
  // in a graph) keeps a valid pointer after a larger call replaces it; the
  // capacity at least doubles at each growth, so the retired buffers
  // together are smaller than the current one
  std::mutex rec_mu;
  uint8_t* scratch_rec = nullptr;
  size_t cap_rec = 0;
  std::vector<void*> retired;
};

std::mutex g_dev_mu;
std::vector<std::unique_ptr<DeviceState>> g_devs;

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  cudaError_t set(int dev) {
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return e;
    if (prev == dev) return cudaSuccess;
    return cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// State of `dev`, created on first use (with `dev` current).
int device_state(int dev, DeviceState** out) {
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (dev >= 0 && static_cast<size_t>(dev) < g_devs.size() && g_devs[dev]) {  // created before
    *out = g_devs[dev].get();
    return FRC_OK;
  }
  int count = 0;
  FRC_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (dev < 0 || dev >= count) return fail(FRC_ERR_INVALID, "device %d out of range (%d devices)", dev, count);
  if (g_devs.size() < static_cast<size_t>(count)) g_devs.resize(count);
  if (!g_devs[dev]) {
    auto s = std::make_unique<DeviceState>();
    s->device = dev;
    DeviceGuard g;
    FRC_CUDA(g.set(dev), "cudaSetDevice");
    FRC_CUDA(cudaDeviceGetAttribute(&s->sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
    FRC_CUDA(cudaMalloc(&s->status, sizeof(uint32_t)), "cudaMalloc(status)");
    FRC_CUDA(cudaMemset(s->status, 0, sizeof(uint32_t)), "cudaMemset(status)");
    FRC_CUDA(cudaMallocHost(&s->status_host, sizeof(uint32_t)), "cudaMallocHost(status)");
    FRC_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    g_devs[dev] = std::move(s);
  }
  *out = g_devs[dev].get();
  return FRC_OK;
}

int current_device_state(DeviceState** out) {
  int dev = 0;
  FRC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  return device_state(dev, out);
}

template <typename T>
int ensure(T** buf, size_t* cap, size_t bytes, const char* what) {
  if (bytes <= *cap) return FRC_OK;
  if (*buf) cudaFree(*buf);
  *buf = nullptr;
  *cap = 0;
  size_t want = bytes < 4096 ? 4096 : bytes;
  want = (want + 255) / 256 * 256;
  FRC_CUDA(cudaMalloc(reinterpret_cast<void**>(buf), want), what);
  *cap = want;
  return FRC_OK;
}

// Host-buffer transfers up to this size go through the pinned staging
// buffer; larger ones are copied directly.
constexpr size_t kPinnedStageMax = size_t(4) << 20;

// Pinned staging of at least `bytes` (grown on demand, freed only on
// growth: a host-buffer call has synchronised before it returns, so no
// transfer from an older buffer is in flight).
int pinned_stage(DeviceState* ds, size_t bytes, uint8_t** out) {
  if (bytes > ds->cap_pinned) {
    size_t want = ds->cap_pinned ? 2 * ds->cap_pinned : (size_t(256) << 10);
    while (want < bytes) want *= 2;
    if (ds->pinned) cudaFreeHost(ds->pinned);
    ds->pinned = nullptr;
    ds->cap_pinned = 0;
    FRC_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ds->pinned), want), "cudaMallocHost(staging)");
    ds->cap_pinned = want;
  }
  *out = ds->pinned;
  return FRC_OK;
}

// Activation-record scratch of at least `bytes` on ds's device (current).
int record_scratch(DeviceState* ds, size_t bytes, uint8_t** out) {
  std::lock_guard<std::mutex> lock(ds->rec_mu);
  if (bytes > ds->cap_rec) {
    size_t want = ds->cap_rec ? 2 * ds->cap_rec : (size_t(2) << 20);
    while (want < bytes) want *= 2;
    void* p = nullptr;
    FRC_CUDA(cudaMalloc(&p, want), "cudaMalloc(activation records)");
    if (ds->scratch_rec) ds->retired.push_back(ds->scratch_rec);
    ds->scratch_rec = static_cast<uint8_t*>(p);
    ds->cap_rec = want;
  }
  *out = ds->scratch_rec;
  return FRC_OK;
}

int launch_gemv_quant(int quant, const frc::GemvRequest& r) {
  cudaError_t e;
  switch (quant) {
    case FRC_Q8_0: e = frc::launch_gemv<frc::kQ8_0>(r); break;
    case FRC_Q4_K: e = frc::launch_gemv<frc::kQ4_K>(r); break;
    case FRC_Q5_K: e = frc::launch_gemv<frc::kQ5_K>(r); break;
    case FRC_Q6_K: e = frc::launch_gemv<frc::kQ6_K>(r); break;
    case FRC_Q1_0: e = frc::launch_gemv<frc::kQ1_0>(r); break;
    default: return fail(FRC_ERR_INVALID, "unsupported quant id %d", quant);
  }
  if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  return FRC_OK;
}

// y (seq, n) = x (seq, k) . W^T on `stream`, all pointers on device `ds`.
int gemv_device(DeviceState* ds, int quant, const uint8_t* w, int64_t n, int64_t k, const float* x, int64_t seq,
                float* y, cudaStream_t stream, uint32_t* status = nullptr) {
  if (!status) status = ds->status;
  if (n == 0) return FRC_OK;
  if (k == 0) {
    FRC_CUDA(cudaMemsetAsync(y, 0, sizeof(float) * n * seq, stream), "cudaMemsetAsync");
    return FRC_OK;
  }
  // more than kMaxGemvBatch columns: the tensor-core prefill GEMM, if the
  // shape suits it (FRC_TC=0 turns it off)
  if (seq > kMaxGemvBatch && frc::opt(frc::options().prefill_tc)) {
    frc::GemvRequest r{};
    r.w = w;
    r.x = x;
    r.y = y;
    r.n = n;
    r.k = static_cast<int>(k);
    r.batch = static_cast<int>(seq);
    r.status = status;
    r.stream = stream;
    r.device = ds->device;
    r.sms = ds->sms;
    r.tc_splits = frc::tc_split_count(quant, n, k, seq, ds->sms);
    int rc = record_scratch(ds, static_cast<size_t>(frc::tc_scratch_bytes(k, n, seq, r.tc_splits)), &r.xrec);
    if (rc != FRC_OK) return rc;
    cudaError_t e;
    switch (quant) {
      case FRC_Q8_0: e = frc::launch_gemm_tc<frc::kQ8_0>(r); break;
      case FRC_Q4_K: e = frc::launch_gemm_tc<frc::kQ4_K>(r); break;
      case FRC_Q5_K: e = frc::launch_gemm_tc<frc::kQ5_K>(r); break;
      case FRC_Q6_K: e = frc::launch_gemm_tc<frc::kQ6_K>(r); break;
      case FRC_Q1_0: e = frc::launch_gemm_tc<frc::kQ1_0>(r); break;
      default: return fail(FRC_ERR_INVALID, "unsupported quant id %d", quant);
    }
    if (e == cudaSuccess) return FRC_OK;
    if (e != cudaErrorNotSupported) return cuda_fail(e, "prefill launch");
    (void)cudaGetLastError();
  }
  // balanced chunks of at most kMaxGemvBatch columns, so a multi-column call
  // never leaves a single column for the batch-1 kernel
  const int64_t nchunk = (seq + kMaxGemvBatch - 1) / kMaxGemvBatch;
  const int64_t csize = (seq + nchunk - 1) / nchunk;
  for (int64_t c0 = 0; c0 < seq; c0 += csize) {
    const int64_t cb = seq - c0 < csize ? seq - c0 : csize;
    frc::GemvRequest r{};
    r.w = w;
    r.x = x + c0 * k;
    r.y = y + c0 * n;
    r.n = n;
    r.k = static_cast<int>(k);
    r.batch = static_cast<int>(cb);
    r.status = status;
    r.stream = stream;
    r.device = ds->device;
    r.sms = ds->sms;
    if (cb > 1) {
      const int rc = record_scratch(ds, static_cast<size_t>(frc::mma_scratch_bytes(k, static_cast<int>(cb))), &r.xrec);
      if (rc != FRC_OK) return rc;
    }
    const int rc = launch_gemv_quant(quant, r);
    if (rc != FRC_OK) return rc;
  }
  return FRC_OK;
}

int dequant_device(DeviceState* ds, int quant, const uint8_t* w, int64_t n_elems, float* out, cudaStream_t stream) {
  frc::DequantRequest r{w, n_elems, out, stream, ds->sms};
  cudaError_t e;
  switch (quant) {
    case FRC_Q8_0: e = frc::launch_dequant<frc::kQ8_0>(r); break;
    case FRC_Q4_K: e = frc::launch_dequant<frc::kQ4_K>(r); break;
    case FRC_Q5_K: e = frc::launch_dequant<frc::kQ5_K>(r); break;
    case FRC_Q6_K: e = frc::launch_dequant<frc::kQ6_K>(r); break;
    case FRC_Q1_0: e = frc::launch_dequant<frc::kQ1_0>(r); break;
    default: return fail(FRC_ERR_INVALID, "unsupported quant id %d", quant);
  }
  if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
  return FRC_OK;
}

// Queue the status readback behind the work on ds->stream, synchronise and
// turn a raised status word into FRC_ERR_DEVICE.
int finish_host_call(DeviceState* ds) {
  FRC_CUDA(cudaMemcpyAsync(ds->status_host, ds->status, sizeof(uint32_t), cudaMemcpyDeviceToHost, ds->stream),
           "status readback");
  FRC_CUDA(cudaStreamSynchronize(ds->stream), "cudaStreamSynchronize");
  if (*ds->status_host != 0) {
    const uint32_t f = *ds->status_host;
    cudaMemsetAsync(ds->status, 0, sizeof(uint32_t), ds->stream);
    cudaStreamSynchronize(ds->stream);
    return fail(FRC_ERR_DEVICE, "kernel reported status 0x%x (a bounded wait ran out)", f);
  }
  return FRC_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// True if [p, p + bytes) is page-locked host memory (cudaHostAlloc,
// cudaHostRegister, torch's pin_memory): both ends are looked up, since a
// contiguous buffer lies inside one allocation.
bool host_pinned(const void* p, size_t bytes) {
  for (const void* q : {p, static_cast<const void*>(static_cast<const uint8_t*>(p) + bytes - 1)}) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    if (a.type != cudaMemoryTypeHost) return false;
  }
  return true;
}

constexpr size_t kHostOutHead = 256;

// The device result buffer of host-buffer matmuls, at least kHostOutHead +
// y_bytes; a new buffer's status word starts at zero (the memset is queued
// before any kernel that may set it).  The old buffer is free: host-buffer
// calls are serialised by ds->mu and synchronise before they return.
int host_out(DeviceState* ds, size_t y_bytes) {
  const size_t want = kHostOutHead + y_bytes;
  if (want <= ds->cap_host_out) return FRC_OK;
  int rc = ensure(&ds->host_out, &ds->cap_host_out, want, "cudaMalloc(result buffer)");
  if (rc) return rc;
  FRC_CUDA(cudaMemsetAsync(ds->host_out, 0, kHostOutHead, ds->stream), "cudaMemsetAsync(result status)");
  return FRC_OK;
}

// Host-buffer matmul on device `dev` with weight bytes already at `w_dev`
// (or, if w_host is non-null, uploaded into scratch first).  The kernels
// report bounded-wait timeouts into the result buffer's own status word,
// which comes back in the same copy as y (FRC_ERR_DEVICE if raised).
int host_matmul(DeviceState* ds, int quant, const uint8_t* w_dev, const uint8_t* w_host, size_t w_bytes, int64_t n,
                int64_t k, const float* x, int64_t seq, float* y) {
  std::lock_guard<std::mutex> lock(ds->mu);
  DeviceGuard g;
  FRC_CUDA(g.set(ds->device), "cudaSetDevice");
  if (w_host) {
    int rc = ensure(&ds->scratch_w, &ds->cap_w, w_bytes, "cudaMalloc(weight scratch)");
    if (rc) return rc;
    if (w_bytes)
      FRC_CUDA(cudaMemcpyAsync(ds->scratch_w, w_host, w_bytes, cudaMemcpyHostToDevice, ds->stream), "weight upload");
    w_dev = ds->scratch_w;
  }
  int rc = ensure(&ds->scratch_x, &ds->cap_x, sizeof(float) * seq * (k ? k : 1), "cudaMalloc(x scratch)");
  if (rc) return rc;
  const size_t xb = sizeof(float) * seq * k, yb = sizeof(float) * seq * n;
  rc = host_out(ds, yb);
  if (rc) return rc;
  uint32_t* status_dev = reinterpret_cast<uint32_t*>(ds->host_out);
  float* y_dev = reinterpret_cast<float*>(ds->host_out + kHostOutHead);
  // page-locked x is the DMA source itself; pageable x goes through the
  // library's pinned staging (one host copy), and so do y and its status
  // word on the way back (one DMA, one host copy)
  const bool x_direct = xb == 0 || host_pinned(x, xb);
  const size_t x_stage_bytes = x_direct ? 0 : (xb + 255) / 256 * 256;
  const bool staged = x_stage_bytes + kHostOutHead + yb <= kPinnedStageMax;
  uint8_t* stage = nullptr;
  if (staged) {
    rc = pinned_stage(ds, x_stage_bytes + kHostOutHead + yb, &stage);
    if (rc) return rc;
  }
  if (xb) {
    const void* src = x;
    if (staged && !x_direct) {
      std::memcpy(stage, x, xb);
      src = stage;
    }
    FRC_CUDA(cudaMemcpyAsync(ds->scratch_x, src, xb, cudaMemcpyHostToDevice, ds->stream), "x upload");
  }
  rc = gemv_device(ds, quant, w_dev, n, k, ds->scratch_x, seq, y_dev, ds->stream, status_dev);
  if (rc) return rc;
  uint8_t* out_stage = staged ? stage + x_stage_bytes : nullptr;
  if (staged) {
    FRC_CUDA(cudaMemcpyAsync(out_stage, ds->host_out, kHostOutHead + yb, cudaMemcpyDeviceToHost, ds->stream),
             "y download");
  } else {
    if (yb) FRC_CUDA(cudaMemcpyAsync(y, y_dev, yb, cudaMemcpyDeviceToHost, ds->stream), "y download");
    FRC_CUDA(cudaMemcpyAsync(ds->status_host, status_dev, sizeof(uint32_t), cudaMemcpyDeviceToHost, ds->stream),
             "status readback");
  }
  FRC_CUDA(cudaStreamSynchronize(ds->stream), "cudaStreamSynchronize");
  const uint32_t f = staged ? *reinterpret_cast<const uint32_t*>(out_stage) : *ds->status_host;
  if (f != 0) {
    cudaMemsetAsync(status_dev, 0, sizeof(uint32_t), ds->stream);
    cudaStreamSynchronize(ds->stream);
    return fail(FRC_ERR_DEVICE, "kernel reported status 0x%x (a bounded wait ran out)", f);
  }
  if (staged && yb) std::memcpy(y, out_stage + kHostOutHead, yb);
  return FRC_OK;
}

int host_dequant(DeviceState* ds, int quant, const uint8_t* w_dev, const uint8_t* w_host, size_t w_bytes,
                 int64_t n_elems, float* out) {
  std::lock_guard<std::mutex> lock(ds->mu);
  DeviceGuard g;
  FRC_CUDA(g.set(ds->device), "cudaSetDevice");
  if (w_host) {
    int rc = ensure(&ds->scratch_w, &ds->cap_w, w_bytes, "cudaMalloc(weight scratch)");
    if (rc) return rc;
    if (w_bytes)
      FRC_CUDA(cudaMemcpyAsync(ds->scratch_w, w_host, w_bytes, cudaMemcpyHostToDevice, ds->stream), "weight upload");
    w_dev = ds->scratch_w;
  }
  int rc = ensure(&ds->scratch_y, &ds->cap_y, sizeof(float) * (n_elems ? n_elems : 1), "cudaMalloc(out scratch)");
  if (rc) return rc;
  rc = dequant_device(ds, quant, w_dev, n_elems, ds->scratch_y, ds->stream);
  if (rc) return rc;
  if (n_elems)
    FRC_CUDA(cudaMemcpyAsync(out, ds->scratch_y, sizeof(float) * n_elems, cudaMemcpyDeviceToHost, ds->stream),
             "dequant download");
  return finish_host_call(ds);
}

// Element count and block count checks of the dequant entry points.  `strict`
// is the _C.cpp rule (element count a multiple of QK); otherwise the NumPy
// rule (ceil(count / QK) blocks, trailing padding dropped, gguf.py:61-75).
int check_dequant(int quant, size_t w_bytes, int64_t n_elems, bool strict) {
  int qk, ts;
  if (!geometry(quant, &qk, &ts)) return fail(FRC_ERR_INVALID, "unsupported quant id %d", quant);
  if (n_elems < 0) return fail(FRC_ERR_INVALID, "%s dequant: negative element count", quant_name(quant));
  if (strict && n_elems % qk != 0)
    return fail(FRC_ERR_INVALID, "%s tensor element count must be a multiple of %d", quant_name(quant), qk);
  const unsigned long long blocks = (unsigned long long)((n_elems + qk - 1) / qk);
  if (w_bytes != blocks * ts)
    return fail(FRC_ERR_INVALID, "%s weight byte size mismatch: expected %llu bytes, got %llu", quant_name(quant),
                blocks * ts, (unsigned long long)w_bytes);
  return FRC_OK;
}

int stateless_matmul(int quant, const float* x, int64_t seq, const uint8_t* w, size_t w_bytes, int64_t n, int64_t k,
                     float* y) {
  int rc = check_matmul(quant, w_bytes, n, k, seq);
  if (rc) return rc;
  if ((w_bytes && !w) || (seq * k && !x) || (seq * n && !y)) return fail(FRC_ERR_INVALID, "null buffer");
  DeviceState* ds;
  rc = current_device_state(&ds);
  if (rc) return rc;
  return host_matmul(ds, quant, nullptr, w, w_bytes, n, k, x, seq, y);
}

int stateless_dequant(int quant, const uint8_t* w, size_t w_bytes, int64_t out_dim, int64_t in_dim, float* out,
                      bool strict) {
  if (out_dim < 0 || in_dim < 0) return fail(FRC_ERR_INVALID, "negative shape");
  const int64_t n_elems = out_dim * in_dim;
  int rc = check_dequant(quant, w_bytes, n_elems, strict);
  if (rc) return rc;
  if ((w_bytes && !w) || (n_elems && !out)) return fail(FRC_ERR_INVALID, "null buffer");
  DeviceState* ds;
  rc = current_device_state(&ds);
  if (rc) return rc;
  return host_dequant(ds, quant, nullptr, w, w_bytes, n_elems, out);
}

// ---- fixed activation-record region for frc_gemv_noalloc -----------------
// The batched tensor-core kernel stages x as 16-bit integer records
// (frc::mma_scratch_bytes(k, batch) bytes).  frc_gemv keeps them in a
// per-device buffer it allocates and grows; frc_gemv_noalloc uses this static
// region instead: the module's own device memory, one instance per device,
// never allocated or freed by the library.  Every call rewrites the records
// it reads, so its contents need no initial value.
constexpr size_t kNoAllocRecordBytes = FRC_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) uint8_t g_noalloc_records[kNoAllocRecordBytes];
// Bounded-wait status of the kernels this entry point launches; zero when the
// module loads (kernels only OR bits into it), read and cleared by
// frc_noalloc_status.
static __device__ uint32_t g_noalloc_status;

struct NoAllocDevice {
  bool ready;
  uint8_t* records;  // device address of g_noalloc_records on this device
  uint32_t* status;
  int sms;
};
constexpr int kNoAllocMaxDevices = 64;
NoAllocDevice g_noalloc[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Device addresses of the static region on the current device, looked up on
// the first call for that device (the host-side names are not device
// addresses).
int noalloc_device(int* dev_out, NoAllocDevice** out) {
  int dev = 0;
  FRC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(FRC_ERR_INVALID, "frc_gemv_noalloc: device %d unsupported", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc[dev];
  if (!d.ready) {
    void* rec = nullptr;
    void* st = nullptr;
    int sms = 0;
    FRC_CUDA(cudaGetSymbolAddress(&rec, g_noalloc_records), "cudaGetSymbolAddress(activation records)");
    FRC_CUDA(cudaGetSymbolAddress(&st, g_noalloc_status), "cudaGetSymbolAddress(status word)");
    FRC_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
    d.records = static_cast<uint8_t*>(rec);
    d.status = static_cast<uint32_t*>(st);
    d.sms = sms;
    d.ready = true;
  }
  *dev_out = dev;
  *out = &d;
  return FRC_OK;
}

}  // namespace

extern "C" {

// Message recorder for the other translation units of the library.
int frc__fail(int code, const char* msg) { return fail(code, "%s", msg); }

int frc_version(char* buf, size_t len) {
  static const char kVersion[] = "frcuda 0.1.0 (sm_100a; Q8_0 Q4_K Q5_K Q6_K Q1_0; TMA-staged GEMV)";
  if (!buf || len == 0) return fail(FRC_ERR_INVALID, "null buffer");
  snprintf(buf, len, "%s", kVersion);
  return FRC_OK;
}

int frc_is_neon(void) { return 0; }

int frc_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return FRC_ERR_INVALID;
  snprintf(buf, len, "%s", g_err.c_str());
  return FRC_OK;
}

int frc_device_count(int* count) {
  if (!count) return fail(FRC_ERR_INVALID, "null pointer");
  *count = 0;
  FRC_CUDA(cudaGetDeviceCount(count), "cudaGetDeviceCount");
  return FRC_OK;
}

int frc_block_geometry(int quant, int* elems_per_block, int* bytes_per_block) {
  int qk, ts;
  if (!geometry(quant, &qk, &ts)) return fail(FRC_ERR_INVALID, "unsupported quant id %d", quant);
  if (elems_per_block) *elems_per_block = qk;
  if (bytes_per_block) *bytes_per_block = ts;
  return FRC_OK;
}

int frc_weight_nbytes(int quant, int64_t n, int64_t k, size_t* nbytes) {
  int qk, ts;
  if (!geometry(quant, &qk, &ts)) return fail(FRC_ERR_INVALID, "unsupported quant id %d", quant);
  if (n < 0 || k < 0 || k % qk) return fail(FRC_ERR_INVALID, "%s: k=%lld is not a multiple of %d", quant_name(quant), (long long)k, qk);
  if (nbytes) *nbytes = static_cast<size_t>(n) * static_cast<size_t>(k / qk) * ts;
  return FRC_OK;
}

int frc_device_status(int device, uint32_t* flags) {
  if (!flags) return fail(FRC_ERR_INVALID, "null pointer");
  DeviceState* ds;
  int rc = device_state(device, &ds);
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(ds->mu);
  DeviceGuard g;
  FRC_CUDA(g.set(device), "cudaSetDevice");
  FRC_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  FRC_CUDA(cudaMemcpy(flags, ds->status, sizeof(uint32_t), cudaMemcpyDeviceToHost), "status read");
  FRC_CUDA(cudaMemset(ds->status, 0, sizeof(uint32_t)), "status clear");
  return FRC_OK;
}

int frc_set_option(int option, int value) {
  frc::Options& o = frc::options();
  switch (option) {
    case FRC_OPT_BATCH1_INT16: o.batch1_int16.store(value ? 1 : 0); return FRC_OK;
    case FRC_OPT_BATCHED_FP32: o.batched_fp32.store(value ? 1 : 0); return FRC_OK;
    case FRC_OPT_PREFILL_TC: o.prefill_tc.store(value ? 1 : 0); return FRC_OK;
    case FRC_OPT_PREFILL_SPLITS:
      if (value < 0) return fail(FRC_ERR_INVALID, "frc_set_option: prefill splits must be >= 0 (got %d)", value);
      o.prefill_splits.store(value);
      return FRC_OK;
    case FRC_OPT_INJECT_OOM: o.inject_oom.store(value ? 1 : 0); return FRC_OK;
    case FRC_OPT_BATCH1_TC:
      if (value < 0 || value > 2) return fail(FRC_ERR_INVALID, "frc_set_option: batch1_tc must be 0, 1 or 2 (got %d)", value);
      o.batch1_tc.store(value);
      return FRC_OK;
    default: return fail(FRC_ERR_INVALID, "frc_set_option: unknown option %d", option);
  }
}

int frc_get_option(int option, int* value) {
  if (!value) return fail(FRC_ERR_INVALID, "null pointer");
  const frc::Options& o = frc::options();
  switch (option) {
    case FRC_OPT_BATCH1_INT16: *value = frc::opt(o.batch1_int16); return FRC_OK;
    case FRC_OPT_BATCHED_FP32: *value = frc::opt(o.batched_fp32); return FRC_OK;
    case FRC_OPT_PREFILL_TC: *value = frc::opt(o.prefill_tc); return FRC_OK;
    case FRC_OPT_PREFILL_SPLITS: *value = frc::opt(o.prefill_splits); return FRC_OK;
    case FRC_OPT_INJECT_OOM: *value = frc::opt(o.inject_oom); return FRC_OK;
    case FRC_OPT_BATCH1_TC: *value = frc::opt(o.batch1_tc); return FRC_OK;
    default: return fail(FRC_ERR_INVALID, "frc_get_option: unknown option %d", option);
  }
}

int frc_batch1_kernel(int quant, int64_t k, int* kind) {
  if (!kind) return fail(FRC_ERR_INVALID, "null pointer");
  int qk, ts;
  if (!geometry(quant, &qk, &ts)) return fail(FRC_ERR_INVALID, "unsupported quant id %d", quant);
  if (k <= 0 || k % qk != 0 || k > (int64_t(1) << 30))
    return fail(FRC_ERR_INVALID, "frc_batch1_kernel: k=%lld is not a positive multiple of %d", (long long)k, qk);
  const frc::Options& o = frc::options();
  frc::Tc1Config c;
  if (frc::opt(o.batch1_int16)) {
    *kind = FRC_B1_INT16;
  } else if ((quant == FRC_Q4_K || quant == FRC_Q5_K) && frc::opt(o.batch1_tc) &&
             frc::tc1_config(ts, static_cast<int>(k), 148, 148, frc::opt(o.batch1_tc) == 2, false, &c)) {
    *kind = FRC_B1_TENSOR_FP32;
  } else {
    *kind = FRC_B1_CUDA_CORE_FP32;
  }
  return FRC_OK;
}

int frc_batch1_plan(int quant, int64_t n, int64_t k, int sms, int64_t* plan) {
  if (!plan) return fail(FRC_ERR_INVALID, "null pointer");
  for (int i = 0; i < FRC_B1_PLAN_LEN; ++i) plan[i] = 0;
  int kind = 0;
  int rc = frc_batch1_kernel(quant, k, &kind);
  if (rc) return rc;
  plan[0] = kind;
  if (n < 1 || n > (int64_t(1) << 40) || sms < 1 || sms > 4096)
    return fail(FRC_ERR_INVALID, "frc_batch1_plan: n must be >= 1 and sms 1..4096");
  if (plan[0] != FRC_B1_TENSOR_FP32) return FRC_OK;
  int qk, ts;
  geometry(quant, &qk, &ts);
  frc::Tc1Config c;
  if (!frc::tc1_config(ts, static_cast<int>(k), n, sms, frc::opt(frc::options().batch1_tc) == 2, false, &c)) {
    plan[0] = FRC_B1_CUDA_CORE_FP32;  // this n does not fit the tensor-core kernel
    return FRC_OK;
  }
  plan[1] = c.nw;
  plan[2] = c.nch;
  plan[3] = c.part_chunks;
  plan[4] = c.split;
  plan[5] = c.split > 1 ? c.ranges : 0;
  plan[6] = c.split > 1 ? static_cast<int64_t>(c.split) * c.ranges : frc::tc1_grid(n, sms);
  plan[7] = c.builders;
  plan[8] = c.nst;
  plan[9] = c.rows_max;
  plan[10] = static_cast<int64_t>(c.smem);
  plan[11] = c.mt;
  return FRC_OK;
}

int frc_gemv(int quant, const void* w_dev, size_t w_bytes, int64_t n, int64_t k, const float* x_dev, int64_t batch,
             float* y_dev, void* stream) {
  int rc = check_matmul(quant, w_bytes, n, k, batch);
  if (rc) return rc;
  if ((w_bytes && !w_dev) || (batch * k && !x_dev) || (batch * n && !y_dev)) return fail(FRC_ERR_INVALID, "null buffer");
  if (!aligned(w_dev, 16)) return fail(FRC_ERR_INVALID, "frc_gemv: weight must be 16-byte aligned");
  if (!aligned(x_dev, 16)) return fail(FRC_ERR_INVALID, "frc_gemv: x must be 16-byte aligned");
  if (!aligned(y_dev, 4)) return fail(FRC_ERR_INVALID, "frc_gemv: y must be 4-byte aligned");
  DeviceState* ds;
  rc = current_device_state(&ds);
  if (rc) return rc;
  return gemv_device(ds, quant, static_cast<const uint8_t*>(w_dev), n, k, x_dev, batch, y_dev,
                     static_cast<cudaStream_t>(stream));
}

int frc_gemv_noalloc(int quant, const void* w_dev, size_t w_bytes, int64_t n, int64_t k, const float* x_dev,
                     int64_t batch, float* y_dev, void* stream) {
  int rc = check_matmul(quant, w_bytes, n, k, batch);
  if (rc) return rc;
  if (batch < 2 || batch > kMaxGemvBatch)
    return fail(FRC_ERR_INVALID, "frc_gemv_noalloc: batch must be 2..%d (got %lld); batch 1 is frc_gemv", kMaxGemvBatch,
                (long long)batch);
  if ((w_bytes && !w_dev) || (batch * k && !x_dev) || (batch * n && !y_dev)) return fail(FRC_ERR_INVALID, "null buffer");
  if (!aligned(w_dev, 16)) return fail(FRC_ERR_INVALID, "frc_gemv_noalloc: weight must be 16-byte aligned");
  if (!aligned(x_dev, 16)) return fail(FRC_ERR_INVALID, "frc_gemv_noalloc: x must be 16-byte aligned");
  if (!aligned(y_dev, 4)) return fail(FRC_ERR_INVALID, "frc_gemv_noalloc: y must be 4-byte aligned");
  const size_t need = static_cast<size_t>(frc::mma_scratch_bytes(k, static_cast<int>(batch)));
  if (need > kNoAllocRecordBytes) {
    int64_t kmax = 0;
    while (static_cast<size_t>(frc::mma_scratch_bytes(kmax + 512, static_cast<int>(batch))) <= kNoAllocRecordBytes)
      kmax += 512;
    return fail(FRC_ERR_INVALID,
                "frc_gemv_noalloc: k=%lld at batch %lld needs %zu bytes of activation records, more than the fixed "
                "%zu (k <= %lld at this batch); use frc_gemv",
                (long long)k, (long long)batch, need, kNoAllocRecordBytes, (long long)kmax);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) return FRC_OK;
  if (k == 0) {
    FRC_CUDA(cudaMemsetAsync(y_dev, 0, sizeof(float) * n * batch, st), "cudaMemsetAsync");
    return FRC_OK;
  }
  int dev = 0;
  NoAllocDevice* d = nullptr;
  rc = noalloc_device(&dev, &d);
  if (rc) return rc;
  frc::GemvRequest r{};
  r.w = static_cast<const uint8_t*>(w_dev);
  r.x = x_dev;
  r.y = y_dev;
  r.n = n;
  r.k = static_cast<int>(k);
  r.batch = static_cast<int>(batch);
  r.status = d->status;
  r.stream = st;
  r.device = dev;
  r.sms = d->sms;
  r.xrec = d->records;
  return launch_gemv_quant(quant, r);
}

int frc_gemv_ex(int quant, int count, const void* const* w_dev, const size_t* w_bytes, const int64_t* n, int64_t k,
                const float* x_dev, const float* x_mul_dev, const float* x_norm_w, float x_norm_eps, int flags,
                float* const* y_dev, void* stream) {
  if (count < 1 || count > 4) return fail(FRC_ERR_INVALID, "frc_gemv_ex: count must be 1..4 (got %d)", count);
  if (!w_dev || !w_bytes || !n || !y_dev) return fail(FRC_ERR_INVALID, "null array");
  if (flags & ~FRC_GEMV_ACCUMULATE) return fail(FRC_ERR_INVALID, "frc_gemv_ex: unknown flags 0x%x", flags);
  int64_t total = 0;
  for (int m = 0; m < count; ++m) {
    int rc = check_matmul(quant, w_bytes[m], n[m], k, 1);
    if (rc) return rc;
    if ((w_bytes[m] && !w_dev[m]) || (n[m] && !y_dev[m])) return fail(FRC_ERR_INVALID, "null buffer");
    if (!aligned(w_dev[m], 16)) return fail(FRC_ERR_INVALID, "frc_gemv_ex: weight %d must be 16-byte aligned", m);
    if (!aligned(y_dev[m], 4)) return fail(FRC_ERR_INVALID, "frc_gemv_ex: y %d must be 4-byte aligned", m);
    total += n[m];
  }
  if ((k && !x_dev) || !aligned(x_dev, 16) || !aligned(x_mul_dev, 16) || !aligned(x_norm_w, 16))
    return fail(FRC_ERR_INVALID, "frc_gemv_ex: x, x_mul and x_norm_w must be 16-byte aligned");
  if (x_mul_dev && x_norm_w) return fail(FRC_ERR_INVALID, "frc_gemv_ex: x_mul and x_norm_w are exclusive");
  if (k == 0 || total == 0) return fail(FRC_ERR_UNSUPPORTED, "frc_gemv_ex: empty shapes");
  DeviceState* ds;
  int rc = current_device_state(&ds);
  if (rc) return rc;
  frc::GemvRequest r{};
  r.k = static_cast<int>(k);
  r.x = x_dev;
  r.batch = 1;
  r.status = ds->status;
  r.stream = static_cast<cudaStream_t>(stream);
  r.device = ds->device;
  r.sms = ds->sms;
  r.nmat = count;
  for (int m = 0; m < count; ++m) {
    r.mat_w[m] = static_cast<const uint8_t*>(w_dev[m]);
    r.mat_y[m] = y_dev[m];
    r.mat_n[m] = n[m];
  }
  r.w = r.mat_w[0];
  r.y = r.mat_y[0];
  r.n = count == 1 ? n[0] : total;
  r.x_mul = x_mul_dev;
  r.x_norm_w = x_norm_w;
  r.x_norm_eps = x_norm_eps;
  r.y_accum = (flags & FRC_GEMV_ACCUMULATE) ? 1 : 0;
  rc = launch_gemv_quant(quant, r);
  if (rc == FRC_OK) return FRC_OK;
  (void)cudaGetLastError();
  return fail(FRC_ERR_UNSUPPORTED, "frc_gemv_ex: no batch-1 fp32 launch for this shape or option (%s)", g_err.c_str());
}

int frc_noalloc_status(int device, uint32_t* flags) {
  if (!flags) return fail(FRC_ERR_INVALID, "null pointer");
  int count = 0;
  FRC_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device < 0 || device >= count) return fail(FRC_ERR_INVALID, "device %d out of range (%d devices)", device, count);
  DeviceGuard g;
  FRC_CUDA(g.set(device), "cudaSetDevice");
  int dev = 0;
  NoAllocDevice* d = nullptr;
  int rc = noalloc_device(&dev, &d);
  if (rc) return rc;
  FRC_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  FRC_CUDA(cudaMemcpy(flags, d->status, sizeof(uint32_t), cudaMemcpyDeviceToHost), "status read");
  FRC_CUDA(cudaMemset(d->status, 0, sizeof(uint32_t)), "status clear");
  return FRC_OK;
}

int frc_gemv_multi(int quant, int count, const void* const* w_dev, const size_t* w_bytes, const int64_t* n,
                   int64_t k, const float* x_dev, int64_t batch, float* const* y_dev, void* stream) {
  if (count < 1 || count > 4) return fail(FRC_ERR_INVALID, "frc_gemv_multi: count must be 1..4 (got %d)", count);
  if (!w_dev || !w_bytes || !n || !y_dev) return fail(FRC_ERR_INVALID, "null array");
  if (batch < 1) return fail(FRC_ERR_INVALID, "frc_gemv_multi: batch must be >= 1");
  for (int m = 0; m < count; ++m) {
    int rc = check_matmul(quant, w_bytes[m], n[m], k, batch);
    if (rc) return rc;
    if ((w_bytes[m] && !w_dev[m]) || (batch * n[m] && !y_dev[m])) return fail(FRC_ERR_INVALID, "null buffer");
    if (!aligned(w_dev[m], 16)) return fail(FRC_ERR_INVALID, "frc_gemv_multi: weight %d must be 16-byte aligned", m);
    if (!aligned(y_dev[m], 4)) return fail(FRC_ERR_INVALID, "frc_gemv_multi: y %d must be 4-byte aligned", m);
  }
  if ((batch * k && !x_dev) || !aligned(x_dev, 16)) return fail(FRC_ERR_INVALID, "frc_gemv_multi: x must be 16-byte aligned");
  DeviceState* ds;
  int rc = current_device_state(&ds);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t total = 0;
  for (int m = 0; m < count; ++m) total += n[m];
  if (batch == 1 && count > 1 && k > 0 && total > 0) {
    frc::GemvRequest r{};
    r.k = static_cast<int>(k);
    r.x = x_dev;
    r.batch = 1;
    r.status = ds->status;
    r.stream = st;
    r.device = ds->device;
    r.sms = ds->sms;
    r.nmat = count;
    for (int m = 0; m < count; ++m) {
      r.mat_w[m] = static_cast<const uint8_t*>(w_dev[m]);
      r.mat_y[m] = y_dev[m];
      r.mat_n[m] = n[m];
    }
    r.n = total;
    rc = launch_gemv_quant(quant, r);
    if (rc == FRC_OK) return FRC_OK;
    g_err.clear();  // not fusable with this shape: one launch per matrix
    (void)cudaGetLastError();
  }
  for (int m = 0; m < count; ++m) {
    rc = gemv_device(ds, quant, static_cast<const uint8_t*>(w_dev[m]), n[m], k, x_dev, batch, y_dev[m], st);
    if (rc) return rc;
  }
  return FRC_OK;
}

int frc_dequant_dev(int quant, const void* w_dev, size_t w_bytes, int64_t n_elems, float* out_dev, void* stream) {
  int rc = check_dequant(quant, w_bytes, n_elems, false);
  if (rc) return rc;
  if ((w_bytes && !w_dev) || (n_elems && !out_dev)) return fail(FRC_ERR_INVALID, "null buffer");
  if (!aligned(w_dev, 2) || !aligned(out_dev, 4)) return fail(FRC_ERR_INVALID, "frc_dequant_dev: misaligned buffer");
  DeviceState* ds;
  rc = current_device_state(&ds);
  if (rc) return rc;
  return dequant_device(ds, quant, static_cast<const uint8_t*>(w_dev), n_elems, out_dev,
                        static_cast<cudaStream_t>(stream));
}

int frc_weight_create(int device, int quant, const void* host, size_t nbytes, int64_t n, int64_t k, frc_weight** out) {
  if (!out) return fail(FRC_ERR_INVALID, "null output handle");
  *out = nullptr;
  int rc = check_matmul(quant, nbytes, n, k, 1);
  if (rc) return rc;
  if (nbytes && !host) return fail(FRC_ERR_INVALID, "null host buffer");
  if (frc::opt(frc::options().inject_oom)) return fail(FRC_ERR_NOMEM, "weight upload: injected allocation failure");
  DeviceState* ds;
  rc = device_state(device, &ds);
  if (rc) return rc;
  DeviceGuard g;
  FRC_CUDA(g.set(device), "cudaSetDevice");
  uint8_t* dev = nullptr;
  const size_t alloc = ((nbytes ? nbytes : 1) + 255) / 256 * 256;
  FRC_CUDA(cudaMalloc(&dev, alloc), "cudaMalloc(weight)");
  if (nbytes) {
    // A pageable cudaMemcpy may return before its DMA has landed, and the
    // kernels that read the weight run on non-blocking streams that do not
    // order behind the legacy stream: copy on this device's stream and wait
    // for it, so the weight is complete when the handle is returned.
    cudaError_t e = cudaMemcpyAsync(dev, host, nbytes, cudaMemcpyHostToDevice, ds->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ds->stream);
    if (e != cudaSuccess) {
      cudaFree(dev);
      return cuda_fail(e, "weight upload");
    }
  }
  frc_weight* w = new frc_weight{device, quant, n, k, nbytes, dev};
  *out = w;
  return FRC_OK;
}

int frc_weight_free(frc_weight* w) {
  if (!w) return FRC_OK;
  DeviceGuard g;
  cudaError_t e = g.set(w->device);
  if (e == cudaSuccess) e = cudaFree(w->dev);
  delete w;
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree(weight)");
  return FRC_OK;
}

int frc_weight_info(const frc_weight* w, const void** dev_ptr, size_t* nbytes, int* quant, int64_t* n, int64_t* k,
                    int* device) {
  if (!w) return fail(FRC_ERR_INVALID, "null weight handle");
  if (dev_ptr) *dev_ptr = w->dev;
  if (nbytes) *nbytes = w->nbytes;
  if (quant) *quant = w->quant;
  if (n) *n = w->n;
  if (k) *k = w->k;
  if (device) *device = w->device;
  return FRC_OK;
}

int frc_weight_matmul(frc_weight* w, const float* x_host, int64_t seq, float* y_host) {
  if (!w) return fail(FRC_ERR_INVALID, "null weight handle");
  if (seq < 1) return fail(FRC_ERR_INVALID, "seq must be >= 1");
  if ((seq * w->k && !x_host) || (seq * w->n && !y_host)) return fail(FRC_ERR_INVALID, "null buffer");
  DeviceState* ds;
  int rc = device_state(w->device, &ds);
  if (rc) return rc;
  return host_matmul(ds, w->quant, w->dev, nullptr, w->nbytes, w->n, w->k, x_host, seq, y_host);
}

int frc_weight_matmul_dev(frc_weight* w, const float* x_dev, int64_t seq, float* y_dev, void* stream) {
  if (!w) return fail(FRC_ERR_INVALID, "null weight handle");
  if (seq < 1) return fail(FRC_ERR_INVALID, "seq must be >= 1");
  if ((seq * w->k && !x_dev) || (seq * w->n && !y_dev)) return fail(FRC_ERR_INVALID, "null buffer");
  if (!aligned(x_dev, 16) || !aligned(y_dev, 4)) return fail(FRC_ERR_INVALID, "misaligned x or y");
  DeviceState* ds;
  int rc = device_state(w->device, &ds);
  if (rc) return rc;
  DeviceGuard g;
  FRC_CUDA(g.set(w->device), "cudaSetDevice");
  return gemv_device(ds, w->quant, w->dev, w->n, w->k, x_dev, seq, y_dev, static_cast<cudaStream_t>(stream));
}

int frc_weight_dequant(frc_weight* w, float* out_host) {
  if (!w) return fail(FRC_ERR_INVALID, "null weight handle");
  if (w->n * w->k && !out_host) return fail(FRC_ERR_INVALID, "null buffer");
  DeviceState* ds;
  int rc = device_state(w->device, &ds);
  if (rc) return rc;
  return host_dequant(ds, w->quant, w->dev, nullptr, w->nbytes, w->n * w->k, out_host);
}

#define FRC_MIRROR(suffix, QUANT, STRICT)                                                                      \
  int frc_matmul_##suffix(const float* x, const uint8_t* w, size_t w_bytes, int64_t n, int64_t k, float* y) {   \
    return stateless_matmul(QUANT, x, 1, w, w_bytes, n, k, y);                                                 \
  }                                                                                                            \
  int frc_matmul_##suffix##_batched(const float* x, int64_t seq, const uint8_t* w, size_t w_bytes, int64_t n,    \
                                    int64_t k, float* y) {                                                     \
    return stateless_matmul(QUANT, x, seq, w, w_bytes, n, k, y);                                               \
  }                                                                                                            \
  int frc_dequant_##suffix(const uint8_t* w, size_t w_bytes, int64_t out_dim, int64_t in_dim, float* out) {      \
    return stateless_dequant(QUANT, w, w_bytes, out_dim, in_dim, out, STRICT);                                 \
  }

FRC_MIRROR(q4_k, FRC_Q4_K, true)
FRC_MIRROR(q8_0, FRC_Q8_0, true)
FRC_MIRROR(q6_k, FRC_Q6_K, true)
FRC_MIRROR(q5_k, FRC_Q5_K, false)
FRC_MIRROR(q1_0, FRC_Q1_0, false)

// ---- fused all-gather across GPUs --------------------------------------------

int frc_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
  if (!dev_ptr || !handle || bytes == 0) return fail(FRC_ERR_INVALID, "frc_ipc_alloc: null argument or zero size");
  *dev_ptr = nullptr;
  void* p = nullptr;
  FRC_CUDA(cudaMalloc(&p, bytes), "cudaMalloc(shared buffer)");
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "cudaIpcGetMemHandle");
  }
  *dev_ptr = p;
  return FRC_OK;
}

int frc_ipc_open(const void* handle, void** dev_ptr) {
  if (!dev_ptr || !handle) return fail(FRC_ERR_INVALID, "frc_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  FRC_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return FRC_OK;
}

int frc_ipc_close(void* dev_ptr) {
  FRC_CUDA(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
  return FRC_OK;
}

int frc_ipc_free(void* dev_ptr) {
  FRC_CUDA(cudaFree(dev_ptr), "cudaFree(shared buffer)");
  return FRC_OK;
}

int frc_gather_create(int world, int rank, void* const* shard_dst, void* const* flags, frc_gather** out) {
  if (!out || !shard_dst || !flags) return fail(FRC_ERR_INVALID, "frc_gather_create: null argument");
  *out = nullptr;
  if (world < 2 || world > frc::kMaxGatherRanks || rank < 0 || rank >= world)
    return fail(FRC_ERR_INVALID, "frc_gather_create: world must be 2..%d and 0 <= rank < world", frc::kMaxGatherRanks);
  for (int r = 0; r < world; ++r)
    if (!shard_dst[r] || !flags[r] || !aligned(shard_dst[r], 4) || !aligned(flags[r], 4))
      return fail(FRC_ERR_INVALID, "frc_gather_create: rank %d pointers null or misaligned", r);
  DeviceState* ds;
  int rc = current_device_state(&ds);
  if (rc) return rc;
  auto g = std::make_unique<frc_gather>();
  g->world = world;
  g->rank = rank;
  g->device = ds->device;
  for (int r = 0; r < world; ++r) {
    g->shard_dst[r] = static_cast<float*>(shard_dst[r]);
    g->flags[r] = static_cast<uint32_t*>(flags[r]);
  }
  FRC_CUDA(cudaMalloc(&g->counters, 2 * sizeof(uint32_t)), "cudaMalloc(gather counters)");
  FRC_CUDA(cudaMemset(g->counters, 0, 2 * sizeof(uint32_t)), "cudaMemset(gather counters)");
  *out = g.release();
  return FRC_OK;
}

int frc_gather_free(frc_gather* g) {
  if (!g) return FRC_OK;
  DeviceGuard guard;
  FRC_CUDA(guard.set(g->device), "cudaSetDevice");
  if (g->counters) cudaFree(g->counters);
  delete g;
  return FRC_OK;
}

int frc_gemv_gather(int quant, int count, const void* const* w_dev, const size_t* w_bytes, const int64_t* n,
                    int64_t k, const float* x_dev, float* const* y_dev, const float* y_base, frc_gather* g,
                    const frc_gather* wait_for, void* stream) {
  if (!g) return fail(FRC_ERR_INVALID, "frc_gemv_gather: null gather");
  if (count < 1 || count > 4) return fail(FRC_ERR_INVALID, "frc_gemv_gather: count must be 1..4 (got %d)", count);
  if (!w_dev || !w_bytes || !n || !y_dev || !y_base) return fail(FRC_ERR_INVALID, "null array");
  int64_t total = 0;
  for (int m = 0; m < count; ++m) {
    int rc = check_matmul(quant, w_bytes[m], n[m], k, 1);
    if (rc) return rc;
    if ((w_bytes[m] && !w_dev[m]) || (n[m] && !y_dev[m])) return fail(FRC_ERR_INVALID, "null buffer");
    if (!aligned(w_dev[m], 16)) return fail(FRC_ERR_INVALID, "frc_gemv_gather: weight %d must be 16-byte aligned", m);
    if (!aligned(y_dev[m], 4) || y_dev[m] < y_base)
      return fail(FRC_ERR_INVALID, "frc_gemv_gather: y %d must be 4-byte aligned and at or above y_base", m);
    total += n[m];
  }
  if ((k && !x_dev) || !aligned(x_dev, 16)) return fail(FRC_ERR_INVALID, "frc_gemv_gather: x must be 16-byte aligned");
  if (k == 0 || total == 0) return fail(FRC_ERR_UNSUPPORTED, "frc_gemv_gather: empty shapes are not gathered");
  DeviceState* ds;
  int rc = current_device_state(&ds);
  if (rc) return rc;
  if (ds->device != g->device) return fail(FRC_ERR_INVALID, "frc_gemv_gather: gather belongs to device %d", g->device);
  frc::GemvRequest r{};
  r.k = static_cast<int>(k);
  r.x = x_dev;
  r.batch = 1;
  r.status = ds->status;
  r.stream = static_cast<cudaStream_t>(stream);
  r.device = ds->device;
  r.sms = ds->sms;
  r.nmat = count;
  for (int m = 0; m < count; ++m) {
    r.mat_w[m] = static_cast<const uint8_t*>(w_dev[m]);
    r.mat_y[m] = y_dev[m];
    r.mat_n[m] = n[m];
  }
  r.w = r.mat_w[0];
  r.y = r.mat_y[0];
  r.n = total;
  r.g_world = g->world;
  r.g_rank = g->rank;
  r.g_ybase = y_base;
  for (int i = 0; i < g->world; ++i) {
    r.g_peer_y[i] = g->shard_dst[i];
    r.g_flags[i] = g->flags[i];
  }
  r.g_done = g->counters;
  r.g_epoch = g->counters + 1;
  if (wait_for) {
    if (wait_for->device != g->device || wait_for->world != g->world)
      return fail(FRC_ERR_INVALID, "frc_gemv_gather: wait_for belongs to another device or world");
    r.w_world = wait_for->world;
    r.w_flags = wait_for->flags[wait_for->rank];
    r.w_epoch = wait_for->counters + 1;
  }
  rc = launch_gemv_quant(quant, r);
  if (rc == FRC_OK) return FRC_OK;
  (void)cudaGetLastError();
  return fail(FRC_ERR_UNSUPPORTED, "frc_gemv_gather: this shape has no fused all-gather path (%s)", g_err.c_str());
}

int frc_gather_wait(frc_gather* g, void* stream) {
  if (!g) return fail(FRC_ERR_INVALID, "frc_gather_wait: null gather");
  DeviceState* ds;
  int rc = current_device_state(&ds);
  if (rc) return rc;
  cudaError_t e = frc::launch_gather_wait(g->flags[g->rank], g->world, g->counters + 1, ds->status,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gather wait launch");
  return FRC_OK;
}

}  // extern "C"
