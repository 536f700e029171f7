/*
 * frcuda.h - C ABI of libfrcuda.so, the B200 (sm_100a) backend for Flatrun's
 * fused GGUF block-dequantise + matrix-vector product.
 *
 * The reference binds this path through pybind11 (module flatrun_native._C,
 * src/flatrun_native/_C.cpp) and selects it through the backend slot
 * (src/flatrun/runtime/backend.py).  Every reference entry point has a
 * counterpart here with plain pointers and sizes, an int status instead of a
 * C++ exception, and no torch or Python types:
 *
 *   reference (_C.cpp)                     here
 *   matmul_q4_k        :99-138             frc_matmul_q4_k
 *   matmul_q4_k_batched:154-197            frc_matmul_q4_k_batched
 *   dequant_q4_k       :47-85              frc_dequant_q4_k
 *   matmul_q8_0        :326-355            frc_matmul_q8_0
 *   matmul_q8_0_batched:199-242            frc_matmul_q8_0_batched
 *   dequant_q8_0       :285-320            frc_dequant_q8_0
 *   matmul_q6_k        :404-433            frc_matmul_q6_k
 *   matmul_q6_k_batched:244-283            frc_matmul_q6_k_batched
 *   dequant_q6_k       :363-398            frc_dequant_q6_k
 *   is_neon            :441-447            frc_is_neon (always 0)
 *   version            :449-451            frc_version
 *   (none: NumPy only, dequant/gguf.py:223, :266)
 *                                          frc_matmul_q5_k[_batched], frc_dequant_q5_k,
 *                                          frc_matmul_q1_0[_batched], frc_dequant_q1_0
 *
 * Those stateless entry points take host buffers, as the reference does, and
 * copy the weight to the GPU on every call.  A backend that calls the same
 * weight many times (the forwarder: once per projection per layer per token)
 * uploads it once with frc_weight_create and then calls frc_weight_matmul,
 * which moves only x and y across PCIe.  frc_gemv / frc_dequant_dev are the
 * stream-ordered device-pointer kernels underneath both.
 *
 * Conventions (the reference's, _C.cpp:105-120 and python/__init__.py:145-153):
 *  - weight: raw GGUF blocks of a row-major (n, k) matrix; row i occupies
 *    bytes [i*(k/QK)*TS, (i+1)*(k/QK)*TS); k must be a multiple of QK.
 *  - x: fp32, (k) or (seq, k) row-major; y: fp32, (n) or (seq, n).
 *  - y[s][i] = sum_j W[i][j] * x[s][j].
 * Every function returns FRC_OK (0) or a nonzero FRC_ERR_*; the message is
 * available from frc_last_error (thread-local).
 */
#ifndef FRCUDA_H
#define FRCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define FRC_OK              0
#define FRC_ERR_INVALID     1  /* bad shape / size / alignment / quant (reference: RuntimeError) */
#define FRC_ERR_CUDA        2  /* a CUDA runtime call failed */
#define FRC_ERR_NOMEM       3  /* device or pinned allocation failed */
#define FRC_ERR_DEVICE      4  /* a kernel reported a fault through its status word (e.g. a bounded wait ran out) */
#define FRC_ERR_UNSUPPORTED 5  /* valid request this build does not implement */

/* quant ids: the GGML type ids of src/flatrun/backend/gguf.py:59-86 */
#define FRC_Q8_0  8
#define FRC_Q4_K 12
#define FRC_Q5_K 13
#define FRC_Q6_K 14
#define FRC_Q1_0 41

/* ---- library / diagnostics -------------------------------------------- */

/* Build identifier (reference: _C.version, _C.cpp:449). */
int frc_version(char* buf, size_t len);
/* Always 0 (reference: _C.is_neon, _C.cpp:441); kept so facades can probe it. */
int frc_is_neon(void);
/* Message of the last failed call on this thread ("" if none). */
int frc_last_error(char* buf, size_t len);
/* Number of visible CUDA devices. */
int frc_device_count(int* count);
/* Elements and bytes per block of a quant (GGML type table, backend/gguf.py:59-86). */
int frc_block_geometry(int quant, int* elems_per_block, int* bytes_per_block);
/* Bytes of an (n, k) weight: n * (k / QK) * TS.  FRC_ERR_INVALID if k % QK != 0. */
int frc_weight_nbytes(int quant, int64_t n, int64_t k, size_t* nbytes);
/* Reads and clears the device status word of `device` (set by kernels whose
 * bounded waits ran out, launched through the device-pointer entry points;
 * the host-buffer calls return FRC_ERR_DEVICE from their own status word
 * instead); *flags == 0 means no fault was recorded. */
int frc_device_status(int device, uint32_t* flags);

/* Library options (no reference counterpart).  Process-wide, read by every
 * later launch; the defaults are the production configuration.
 *  FRC_OPT_BATCH1_INT16   0 (default): batch 1 keeps x in fp32 and forms every
 *                         product in fp32, the reference's arithmetic
 *                         (kernels/q4_k.h:153-184); 1: x is quantised per
 *                         64-element unit to a 16-bit integer grid and the
 *                         products run on dp4a (~3e-5 relative error).
 *  FRC_OPT_BATCHED_FP32   0 (default): batch 2..16 on the int8 tensor-core
 *                         kernel; 1: on the fp32 CUDA-core kernel.
 *  FRC_OPT_PREFILL_TC     1 (default): batches above 16 on the tcgen05 GEMM;
 *                         0: in chunks of at most 16 columns.
 *  FRC_OPT_PREFILL_SPLITS 0 (default): k-splits of the prefill GEMM chosen from
 *                         the shape; n > 0: n splits (clamped to 1..16).
 *  FRC_OPT_INJECT_OOM     1: frc_weight_create fails with FRC_ERR_NOMEM before
 *                         any CUDA call (a test of the error path); default 0.
 *  FRC_OPT_BATCH1_TC      1 (default): batch-1 Q4_K and Q5_K with x in fp32
 *                         run on the tensor cores (weights as exact fp16
 *                         integers q * sc, x as an exact sum of three fp16
 *                         terms, fp32 accumulation); rows whose activation
 *                         fragments do not fit one CTA's shared memory run
 *                         in parts of k on thread-block clusters, one part
 *                         per CTA (up to 8 parts); 2: also rows of more
 *                         than two parts on one CTA without builder warps
 *                         (reached only without clusters); 0: on the
 *                         CUDA-core fp32 kernel. */
#define FRC_OPT_BATCH1_INT16   1
#define FRC_OPT_BATCHED_FP32   2
#define FRC_OPT_PREFILL_TC     3
#define FRC_OPT_PREFILL_SPLITS 4
#define FRC_OPT_INJECT_OOM     5
#define FRC_OPT_BATCH1_TC      6
int frc_set_option(int option, int value);
int frc_get_option(int option, int* value);
/* The batch-1 kernel a launch of (quant, k) runs under the current options
 * (no reference counterpart): FRC_B1_CUDA_CORE_FP32 (x in fp32, fp32 FMAs),
 * FRC_B1_TENSOR_FP32 (x in fp32 as three exact fp16 terms, tensor-core
 * products, fp32 accumulation) or FRC_B1_INT16 (16-bit grid, dp4a). */
#define FRC_B1_CUDA_CORE_FP32 0
#define FRC_B1_TENSOR_FP32    1
#define FRC_B1_INT16          2
int frc_batch1_kernel(int quant, int64_t k, int* kind);
/* The batch-1 launch plan of an (n, k) matrix on a device of `sms` SMs under
 * the current options, computed on the host without launching anything (no
 * reference counterpart; for diagnostics and for tests that need no GPU).
 * plan[FRC_B1_PLAN_LEN]: [0] the kernel (FRC_B1_*); for FRC_B1_TENSOR_FP32
 * also [1] compute warps (super-blocks per chunk), [2] chunks per row,
 * [3] chunks per part of k, [4] CTAs per cluster (1: one CTA per row range,
 * every part; s > 1: one part per CTA), [5] row ranges (clusters) wanted
 * when split, [6] CTAs, [7] builder warps, [8] shared-memory stages,
 * [9] most rows one CTA or cluster holds, [10] dynamic shared memory bytes,
 * [11] 16-row MMA tiles per warp. */
#define FRC_B1_PLAN_LEN 12
int frc_batch1_plan(int quant, int64_t n, int64_t k, int sms, int64_t* plan);

/* ---- stream-ordered device-pointer kernels ------------------------------ *
 * No synchronisation: the work is enqueued on `stream` (a cudaStream_t;
 * NULL = legacy default stream) of the current device.  w_dev must be
 * 16-byte aligned.  frc_gemv computes y_dev (batch, n) from x_dev (batch, k),
 * batch >= 1: batch 1 on the fp32-activation kernel (FRC_OPT_BATCH1_INT16
 * selects the dp4a one), 2..16 on the int8 tensor-core kernel, more (prefill) on the tcgen05 GEMM with fp16 operands and fp32
 * accumulation (where the row length allows its tensor view; otherwise in
 * chunks of at most 16 columns).  For batch >= 2 x is first staged (as
 * 16-bit integer records, or as fp16) in a per-device buffer the library
 * owns; it is allocated on the first such call and grown (old buffers are
 * kept until exit) when a later call needs more.  Calls with batch >= 2 on
 * one device share it, so they must not overlap in time across streams. */
int frc_gemv(int quant, const void* w_dev, size_t w_bytes, int64_t n, int64_t k,
             const float* x_dev, int64_t batch, float* y_dev, void* stream);
/* Batched GEMV that allocates no device memory (no counterpart in the
 * reference).  Same arguments and result as frc_gemv for 2 <= batch <= 16,
 * but the activation records live in a fixed region of
 * FRC_NOALLOC_SCRATCH_BYTES of the library's own static device memory (one
 * per device) instead of a buffer allocated on demand.  It serves callers
 * that cannot allocate once they run: an engine that has committed all of
 * HBM to weights and KV cache, a device-memory pool policy that forbids
 * cudaMalloc after start-up, or a decode loop that cannot take the
 * device-wide synchronisation cudaMalloc/cudaFree may cause.
 * Limit: the records take ceil(k/512) * C * 1600 bytes, C = 4, 8 or 16 (batch
 * rounded up to one of those), i.e. k <= 167424 at batch <= 4, 83456 at <= 8
 * and 41472 at <= 16; larger k, batch 1 or batch > 16 return FRC_ERR_INVALID
 * with a message.  The first call on each device (with that
 * device current) looks up the region's device address; make that first call
 * before any stream capture.  No memory needs to start at zero: each call
 * rewrites the records it reads.  All calls on one device share the region,
 * so two calls that can overlap in time (streams without ordering between
 * them) race and give wrong results.  A bounded wait that runs out sets a bit
 * in this entry point's own status word (also static device memory) and y is
 * then incomplete: frc_noalloc_status reads and clears that word. */
#define FRC_NOALLOC_SCRATCH_BYTES 2097152
int frc_gemv_noalloc(int quant, const void* w_dev, size_t w_bytes, int64_t n, int64_t k,
                     const float* x_dev, int64_t batch, float* y_dev, void* stream);
/* Reads and clears the status word of frc_gemv_noalloc on `device`, after
 * waiting for the device's queued work; *flags == 0 means every call so far
 * completed.  Allocates nothing.  (No reference counterpart.) */
int frc_noalloc_status(int device, uint32_t* flags);
/* One launch for up to 4 weights of the same quant and k that share x
 * (q/k/v, or gate/up, of a layer): y_dev[m] (batch, n[m]) = x . W_m^T.  At
 * batch 1 the rows of all matrices form one row space of a single kernel
 * launch; otherwise, or when the shape does not allow it, one launch per
 * matrix.  Same alignment rules as frc_gemv.  (No reference counterpart: the
 * reference dispatches one projection per call, flatrun/model/qwen2.py:1510-1519.) */
int frc_gemv_multi(int quant, int count, const void* const* w_dev, const size_t* w_bytes, const int64_t* n,
                   int64_t k, const float* x_dev, int64_t batch, float* const* y_dev, void* stream);
/* Batch-1 launch of up to 4 weights of the same quant and k sharing x (as
 * frc_gemv_multi) with two options of the fp32-activation kernel, for a
 * device-resident decoder step (no reference counterpart: the reference
 * forwarder does both in NumPy, flatrun/model/qwen2.py:1617-1646, :1690-1751):
 *  - x_mul_dev != NULL: the activations are silu(x) * x_mul elementwise,
 *    silu(g) = g / (1 + exp(-g)) evaluated as (1 / (1 + exp(-g))) * g, so a
 *    gate and an up projection feed the down projection with no SwiGLU pass;
 *  - x_norm_w != NULL: the activations are RMSNorm(x) * x_norm_w,
 *    x * (1 / sqrt(mean(x^2) + x_norm_eps)) * w (qwen2.py:365-378), the mean
 *    taken over the whole row inside the launch, so no separate norm pass
 *    (exclusive with x_mul);
 *  - flags & FRC_GEMV_ACCUMULATE: y += W x instead of y = W x (a residual
 *    stream).
 * FRC_ERR_UNSUPPORTED when the batch-1 int16 option is set or the row is
 * too long for one CTA. */
#define FRC_GEMV_ACCUMULATE 1
int frc_gemv_ex(int quant, int count, const void* const* w_dev, const size_t* w_bytes, const int64_t* n,
                int64_t k, const float* x_dev, const float* x_mul_dev, const float* x_norm_w, float x_norm_eps,
                int flags, float* const* y_dev, void* stream);

/* ---- device-resident decoder step ----------------------------------------- *
 * The operators of a Qwen2/Llama decode token around the projections, so a
 * whole token runs on the GPU (stream-ordered, no synchronisation, graph
 * capturable).  They restate the reference forwarder's NumPy steps
 * (flatrun/model/qwen2.py): RMSNorm :365-378, q/k/v bias + rotate-half RoPE
 * + KV append :1527-1595 (tables :398-476), GQA attention :1597-1614,
 * embedding row :2153-2159.  The token's position is read from device
 * memory (pos_dev, one int) so the same launches replay for every token;
 * frc_pos_advance increments it.
 *  frc_rmsnorm: out[r] = x[r] * (1 / sqrt(mean(x[r]^2) + eps)) * w, rows of n.
 *  frc_rope_append: qkv = [q (nh*hd) | k (nkv*hd) | v (nkv*hd)] of one token;
 *    adds `bias` (same layout, may be NULL), rotates q in place and k at
 *    position *pos_dev with cos/sin tables [max_pos][hd/2], writes k and v to
 *    row *pos_dev of the caches ([max_pos][nkv][hd]).
 *  frc_attention_decode: one query token (q, nh*hd, rotated) over cache rows
 *    0..*pos_dev: softmax(q.k * scale) . v per head, query head h reading KV
 *    head h / (nh/nkv); positions split into `splits` ranges (flash
 *    decoding) whose partials (frc_attention_workspace floats in `part`) are
 *    merged into out (nh*hd).  hd 64 or 128, nh/nkv <= 8, splits <= 1024.
 *  frc_argmax: index of the largest of n floats into *out_dev (the lowest
 *    index among ties, as np.argmax); `workspace` holds
 *    frc_argmax_workspace bytes, zeroed before the first call (the kernel
 *    leaves it ready for the next).
 *  frc_embed_row: row *tok_dev of a (vocab, n) table into out: quant 0 for
 *    fp32 rows, or a GGUF quant id (dequantised bit-exactly). */
int frc_rmsnorm(const float* x, const float* w, int64_t rows, int64_t n, float eps, float* out, void* stream);
int frc_rope_append(float* qkv, const float* bias, int nh, int nkv, int hd, const float* cos_table,
                    const float* sin_table, const int* pos_dev, float* k_cache, float* v_cache, void* stream);
int frc_attention_workspace(int nh, int hd, int splits, size_t* floats);
int frc_attention_decode(const float* q, const float* k_cache, const float* v_cache, const int* pos_dev, int nh,
                         int nkv, int hd, float scale, int splits, float* part, float* out, void* stream);
int frc_argmax_workspace(int64_t n, size_t* bytes);
int frc_argmax(const float* x, int64_t n, int* out_dev, void* workspace, void* stream);
int frc_embed_row(int quant, const void* table, int64_t n, const int* tok_dev, float* out, void* stream);
int frc_pos_advance(int* pos_dev, void* stream);

/* ---- row-sharded projections: all-gather fused into the GEMV ----------- *
 * No reference counterpart: the reference runs on one CPU.  One process per
 * GPU; rank r owns a contiguous row range of every projection and computes
 * its y shard; the shards are assembled in every rank's gathered buffer by
 * the GEMV itself, which stores each y value also into every rank's buffer
 * (over NVLink peer mappings), so no separate collective runs.
 * Set-up: each rank allocates its gathered buffer and a flag array of
 * `world` 32-bit words with frc_ipc_alloc (zeroed), exchanges the handles
 * (FRC_IPC_HANDLE_BYTES each, e.g. through torch.distributed) and maps its
 * peers' buffers with frc_ipc_open.  frc_gather_create takes, for every rank
 * r, the address of this rank's shard inside r's gathered buffer and r's
 * flag array (peer mappings, or this rank's own pointers for r == rank).
 * Per use: frc_gemv_gather (batch 1: the fused launch of up to four
 * matrices sharing x, as frc_gemv_multi; y_dev[m] are this rank's outputs
 * and y_base the address that offsets into the gathered buffers are taken
 * from).  Its result is complete on every rank once a later kernel has
 * waited for it: pass that gather as `wait_for` to the next frc_gemv_gather
 * on the stream (the GEMV waits before reading x, which may be the gathered
 * buffer), or call frc_gather_wait (a one-block kernel).  Waits are bounded
 * at 1 s; a timeout sets a bit in the device status word.  Every rank must
 * issue the same sequence of gathers.  frc_gemv_gather returns
 * FRC_ERR_UNSUPPORTED for shapes without the fused path (callers then use a
 * collective).  world <= 8. */
#define FRC_IPC_HANDLE_BYTES 64
int frc_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
int frc_ipc_open(const void* handle, void** dev_ptr);
int frc_ipc_close(void* dev_ptr);
int frc_ipc_free(void* dev_ptr);
typedef struct frc_gather frc_gather;
int frc_gather_create(int world, int rank, void* const* shard_dst, void* const* flags, frc_gather** out);
int frc_gather_free(frc_gather* g);
int frc_gemv_gather(int quant, int count, const void* const* w_dev, const size_t* w_bytes, const int64_t* n,
                    int64_t k, const float* x_dev, float* const* y_dev, const float* y_base, frc_gather* g,
                    const frc_gather* wait_for, void* stream);
int frc_gather_wait(frc_gather* g, void* stream);
/* Bit-exact dequantisation of n_elems elements (ceil(n_elems/QK) blocks) into
 * out_dev (n_elems floats), matching the reference NumPy decoders
 * (dequant/gguf.py) bit for bit. */
int frc_dequant_dev(int quant, const void* w_dev, size_t w_bytes, int64_t n_elems,
                    float* out_dev, void* stream);

/* ---- device-resident weights (upload once, call many times) ------------- */
typedef struct frc_weight frc_weight;

/* Copies `nbytes` of raw GGUF blocks from host memory to `device`.  The
 * host buffer is not retained. */
int frc_weight_create(int device, int quant, const void* host, size_t nbytes,
                      int64_t n, int64_t k, frc_weight** out);
int frc_weight_free(frc_weight* w);
/* Device address and size of the uploaded blocks. */
int frc_weight_info(const frc_weight* w, const void** dev_ptr, size_t* nbytes,
                    int* quant, int64_t* n, int64_t* k, int* device);
/* y_host (seq, n) = x_host (seq, k) . W^T with host buffers: copies x in,
 * runs frc_gemv (seq <= 16) or the batched prefill path (seq > 16), copies y
 * out and synchronises.  seq >= 1.  Page-locked x is copied from directly;
 * the call's status word comes back with y, and a bounded wait that ran out
 * makes the call return FRC_ERR_DEVICE.  (Reference: matmul_*[_batched].) */
int frc_weight_matmul(frc_weight* w, const float* x_host, int64_t seq, float* y_host);
/* Device-pointer variant on a caller stream; no synchronisation. */
int frc_weight_matmul_dev(frc_weight* w, const float* x_dev, int64_t seq, float* y_dev,
                          void* stream);
/* Dequantise the whole weight to out_host (n*k floats).  (Reference: dequant_*.) */
int frc_weight_dequant(frc_weight* w, float* out_host);

/* ---- stateless host-buffer mirrors of flatrun_native._C ----------------- *
 * w_bytes must equal n*(k/QK)*TS (reference: "weight byte size mismatch").  */
int frc_matmul_q4_k(const float* x, const uint8_t* w, size_t w_bytes, int64_t n, int64_t k, float* y);
int frc_matmul_q4_k_batched(const float* x, int64_t seq, const uint8_t* w, size_t w_bytes,
                            int64_t n, int64_t k, float* y);
int frc_dequant_q4_k(const uint8_t* w, size_t w_bytes, int64_t out_dim, int64_t in_dim, float* out);
int frc_matmul_q8_0(const float* x, const uint8_t* w, size_t w_bytes, int64_t n, int64_t k, float* y);
int frc_matmul_q8_0_batched(const float* x, int64_t seq, const uint8_t* w, size_t w_bytes,
                            int64_t n, int64_t k, float* y);
int frc_dequant_q8_0(const uint8_t* w, size_t w_bytes, int64_t out_dim, int64_t in_dim, float* out);
int frc_matmul_q6_k(const float* x, const uint8_t* w, size_t w_bytes, int64_t n, int64_t k, float* y);
int frc_matmul_q6_k_batched(const float* x, int64_t seq, const uint8_t* w, size_t w_bytes,
                            int64_t n, int64_t k, float* y);
int frc_dequant_q6_k(const uint8_t* w, size_t w_bytes, int64_t out_dim, int64_t in_dim, float* out);
int frc_matmul_q5_k(const float* x, const uint8_t* w, size_t w_bytes, int64_t n, int64_t k, float* y);
int frc_matmul_q5_k_batched(const float* x, int64_t seq, const uint8_t* w, size_t w_bytes,
                            int64_t n, int64_t k, float* y);
int frc_dequant_q5_k(const uint8_t* w, size_t w_bytes, int64_t out_dim, int64_t in_dim, float* out);
int frc_matmul_q1_0(const float* x, const uint8_t* w, size_t w_bytes, int64_t n, int64_t k, float* y);
int frc_matmul_q1_0_batched(const float* x, int64_t seq, const uint8_t* w, size_t w_bytes,
                            int64_t n, int64_t k, float* y);
int frc_dequant_q1_0(const uint8_t* w, size_t w_bytes, int64_t out_dim, int64_t in_dim, float* out);

#ifdef __cplusplus
}
#endif

#endif /* FRCUDA_H */
