/*
 * bw_ops.h — C ABI of the B200 (sm_100a) W8A16 / LoRA-delta operator library.
 *
 * Every entry point takes plain device pointers, element counts, row strides
 * (in elements) and a CUDA stream (cudaStream_t passed as void*; NULL = the
 * legacy default stream).  Nothing allocates device memory: outputs and
 * workspaces are supplied by the caller.  Every function returns a status
 * code (BW_OK == 0); bw_status_string() names it and bw_last_error() gives
 * the calling thread's detail message for the last failure.
 *
 * Kernels run asynchronously on the given stream.  A kernel whose bounded
 * internal wait expires records a device-side status instead of hanging;
 * read it with bw_device_status().
 *
 * Library: libbw_ops.so (built for sm_100a only).
 */
#ifndef BW_OPS_H
#define BW_OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define BW_DTYPE_F16 0
#define BW_DTYPE_BF16 1
#define BW_DTYPE_F32 2

/* status codes */
#define BW_OK 0
#define BW_ERR_INVALID_ARGUMENT 1 /* bad pointer / shape / dtype / stride */
#define BW_ERR_WORKSPACE 2        /* workspace missing or too small */
#define BW_ERR_CUDA 3             /* a CUDA runtime call failed (launch, config) */
#define BW_ERR_DEVICE_TIMEOUT 4   /* a kernel's bounded wait expired (device status) */
#define BW_ERR_UNSUPPORTED 5      /* device is not sm_100 or feature unavailable */

const char* bw_status_string(int status);
/* Detail of the calling thread's last non-OK return (empty string if none). */
const char* bw_last_error(void);
/* Library version, major*10000 + minor*100 + patch. */
int bw_version(void);

/*
 * Per-output-channel symmetric int8 quantisation.
 * Replaces quantize_weight_int8, src/blackwell_ops/kernels/int8_gemm.py:63-68.
 *   w      [n, k] row stride ldw, dtype w_dtype (F16 | BF16 | F32)
 *   q      [n, k] int8, row stride ldq
 *   scale  [n] in w_dtype
 * scale = dt(max|w_row| clamped >= 1e-8, / 127); q = clamp(rne(dt(w/scale)), +-127).
 * Bit-exact with the reference.  n == 0 is a no-op; k must be >= 1.
 */
int bw_quantize_rowwise_int8(const void* w, int w_dtype, int64_t n, int64_t k, int64_t ldw,
                             int8_t* q, int64_t ldq, void* scale, void* stream);

/*
 * W8A16 GEMM: y[m, n] = dt( (sum_k x[m,k] * w[n,k]) * scale[n] ), fp32 accumulation.
 * Replaces int8_gemm, src/blackwell_ops/kernels/int8_gemm.py:71-107 (kernel :15-60).
 *   x      [m, k] x_dtype (F16 | BF16), row stride ldx
 *   w      [n, k] int8, row stride ldw
 *   scale  [n] scale_dtype (F16 | BF16 | F32)
 *   y      [m, n] x_dtype, row stride ldy
 *   workspace: device memory of bw_w8a16_gemm_workspace_size() bytes whose
 *   first bw_w8a16_gemm_workspace_zeroed_bytes() bytes are zero before the
 *   first call (split-K / stream-K tile counters; every successful call leaves
 *   them zero).  The zeroed prefix has the same size for every shape, so one
 *   workspace sized for the largest shape serves calls of any shapes.
 * Calls that share a workspace must not overlap on the GPU.
 */
size_t bw_w8a16_gemm_workspace_size(int64_t m, int64_t n, int64_t k);
size_t bw_w8a16_gemm_workspace_zeroed_bytes(int64_t m, int64_t n, int64_t k);
int bw_w8a16_gemm(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                  const void* scale, int scale_dtype, void* y, int64_t ldy, int64_t m, int64_t n,
                  int64_t k, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Fused gate/up W8A16 GEMM with the SwiGLU epilogue, one launch:
 *   y[m, n] = dt( silu(g) * u ),  g = dt(x @ (w_gate * scale_gate)^T)[m, n],
 *                                 u = dt(x @ (w_up * scale_up)^T)[m, n],  silu(g) = g / (1 + expf(-g)),
 * i.e. swiglu(int8_gemm(x, w_gate, s_gate), int8_gemm(x, w_up, s_up)) with the silu in fp32.
 * Replaces that composition: int8_gemm (src/blackwell_ops/kernels/int8_gemm.py:71-107) twice and
 * swiglu (src/blackwell_ops/cuda/basic_ops.cu:112-122, cuda/__init__.py:74).
 *   w_gate, w_up [n, k] int8 with the same row stride ldw; scale_gate, scale_up [n] scale_dtype;
 *   x, y as for bw_w8a16_gemm.  Workspace: bw_w8a16_gemm_swiglu_workspace_size(m, n, k) bytes,
 *   same zeroing rule as bw_w8a16_gemm (zeroed prefix: bw_w8a16_gemm_workspace_zeroed_bytes of any
 *   split plan, 4096 bytes).
 */
size_t bw_w8a16_gemm_swiglu_workspace_size(int64_t m, int64_t n, int64_t k);
int bw_w8a16_gemm_swiglu(const void* x, int x_dtype, int64_t ldx, const int8_t* w_gate, const int8_t* w_up,
                         int64_t ldw, const void* scale_gate, const void* scale_up, int scale_dtype, void* y,
                         int64_t ldy, int64_t m, int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * W8A16 GEMM that allocates nothing.  No counterpart in the reference: it exists
 * for callers that cannot provide device memory, such as a serving runtime whose
 * memory manager owns the whole GPU and refuses allocations from plug-ins, or a
 * foreign-language binding with no access to a CUDA allocator.
 * Same arguments and result as bw_w8a16_gemm minus the workspace: the split-K
 * scratch is a fixed array inside libbw_ops.so of
 * bw_w8a16_gemm_static_scratch_bytes() (8 MiB), one per GPU that loads the
 * library, held until the process exits.
 *  - The first call on a device looks up the array's device address (set-up);
 *    make that first call before any stream capture.
 *  - Shapes whose scratch need (bw_w8a16_gemm_workspace_size) exceeds the array
 *    are rejected with BW_ERR_WORKSPACE.
 *  - Every call shares the array and clears its counter prefix first (an async
 *    memset on `stream`): calls that overlap on the GPU race.
 */
size_t bw_w8a16_gemm_static_scratch_bytes(void);
int bw_w8a16_gemm_noalloc(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                          const void* scale, int scale_dtype, void* y, int64_t ldy, int64_t m,
                          int64_t n, int64_t k, void* stream);

/*
 * Grouped W8A16 GEMM: y_i = x @ (w_i * scale_i)^T for count <= 4 GEMMs that share x [m, k]
 * (e.g. a layer's q/k/v or gate/up projections), in one persistent launch whose schedule spans
 * the union of their output tiles, so small projections stream as one weight walk instead of one
 * latency-bound launch each.  w_i [n_i, k] int8 (row stride ldw[i]), scale_i [n_i] (scale_dtype for
 * all), y_i [m, ldy[i]] in x's dtype.  Workspace: bw_w8a16_gemm_grouped_workspace_size bytes, its
 * first 4 KB zero, as for bw_w8a16_gemm.  Layouts TMA cannot address run as separate bw_w8a16_gemm
 * calls.  No reference counterpart (the reference calls int8_gemm once per projection).
 */
size_t bw_w8a16_gemm_grouped_workspace_size(int64_t m, const int64_t* n, int count, int64_t k);
int bw_w8a16_gemm_grouped(const void* x, int x_dtype, int64_t ldx, int count, const int8_t* const* w,
                          const int64_t* ldw, const void* const* scale, int scale_dtype, void* const* y,
                          const int64_t* ldy, const int64_t* n, int64_t m, int64_t k, void* workspace,
                          size_t workspace_bytes, void* stream);

/*
 * Column-parallel N-split W8A16 GEMM with the all-gather fused into the
 * epilogue (the north star's N-split; the reference has no multi-GPU path).
 * Rank `rank` of `world` (<= 8) holds w rows [0, n) of its shard; rank p's
 * output columns are [col0 + (p - rank) n, col0 + (p - rank + 1) n) of y
 * [m, ldy], a plain device buffer of this rank.  Each output tile this rank
 * computes is stored into y and, as 8-byte {2 outputs, call epoch} words, into
 * every peer's signal pad (plain stores over NVLink, no fence); the kernel
 * copies its peers' words into y as they arrive, so y holds all world * n
 * columns when the kernel ends.  signal_ranks is a host array of `world`
 * device pointers valid in this process (e.g. a symmetric-memory buffer's peer
 * addresses), 16-byte aligned, each pad signal_bytes >=
 * bw_w8a16_gemm_allgather_signal_bytes(m, n, world) long, zero before the
 * first call and not shared with other users.  m <= 256.  Every rank must make
 * the same calls in the same order with the same m, n, k (pad the last rank's
 * shard to the others' row count), on GPUs with the same SM count: the ranks
 * share one tile schedule.  Waits for peers are bounded (a timeout shows in
 * bw_device_status; the pads must then be zeroed on every rank before the
 * next call).  Workspace: bw_w8a16_gemm_allgather_workspace_size bytes, first
 * bw_w8a16_gemm_workspace_zeroed_bytes zero, as for bw_w8a16_gemm.  x and w
 * must be TMA-addressable.
 */
size_t bw_w8a16_gemm_allgather_workspace_size(int64_t m, int64_t n, int64_t k);
size_t bw_w8a16_gemm_allgather_signal_bytes(int64_t m, int64_t n, int world);
int bw_w8a16_gemm_allgather(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                            const void* scale, int scale_dtype, void* y, int64_t ldy, int64_t col0,
                            int64_t m, int64_t n, int64_t k, void* const* signal_ranks,
                            size_t signal_bytes, int world, int rank, void* workspace,
                            size_t workspace_bytes, void* stream);

/*
 * Stream-K schedule introspection (host only, no device work; used by the tests to check the
 * schedule code the GEMM kernel itself runs).  A plan of `tiles` tiles of `kblocks` k-blocks over
 * `grid` CTAs (kblocks * tiles >= grid, kblocks * tiles * grid < 2^31):
 *   _walk:   CTA `cta`'s segments as {tile, first k-block, k-blocks, slot} quadruples into segs
 *            (at most max_segs); returns their count, -1 on invalid arguments.
 *   _start:  first flattened k-block of CTA `cta` (cta == grid: the end of the work).
 *   _owner:  the CTA whose range holds flattened k-block x.
 *   _pieces: tile `tile`'s first contributor, number of contributors and the first contributor's
 *            piece slot, into loc[0..2].
 */
int bw_debug_streamk_walk(int64_t kblocks, int64_t tiles, int grid, int cta, int32_t* segs, int max_segs);
int64_t bw_debug_streamk_start(int64_t kblocks, int64_t tiles, int grid, int cta);
int bw_debug_streamk_owner(int64_t kblocks, int64_t tiles, int grid, int64_t x);
int bw_debug_streamk_pieces(int64_t kblocks, int64_t tiles, int grid, int tile, int32_t* loc);

/*
 * LoRA delta: delta[n, k] = fp16( fp32(sum_j b[n,j] * a[j,k]) * scaling ).
 * Replaces lora_delta (src/blackwell_ops/cuda/lora_ops.cu:43-60) and
 * lora_delta_tiled (src/blackwell_ops/cuda/lora_tiled.cu:88-103).
 *   a [r, k] fp16 contiguous, b [n, r] fp16 contiguous, delta [n, k] fp16 contiguous.
 */
int bw_lora_delta(const void* a, const void* b, void* delta, int64_t n, int64_t k, int64_t r,
                  float scaling, void* stream);

/*
 * Reference-order ("exact") LoRA delta and merge on the CUDA cores: each output is the reference
 * kernels' own j-ordered fp32 accumulation (lora_ops.cu:16-27) rounded as they round it, so delta,
 * the merged weight and a requantisation of it (bw_quantize_rowwise_int8) equal the reference
 * pipeline bit for bit.  Same arguments as bw_lora_delta / bw_lora_merge; slower than the
 * tensor-core path (r fp32 FMAs per output on the CUDA cores), whose sums are within one fp16 ulp.
 */
int bw_lora_delta_exact(const void* a, const void* b, void* delta, int64_t n, int64_t k, int64_t r,
                        float scaling, void* stream);
int bw_lora_merge_exact(const void* w, int64_t ldw, const void* a, const void* b, float scaling,
                        void* w_out, int64_t ldo, int64_t n, int64_t k, int64_t r, void* stream);

/*
 * In-place merge w[i] = fp16(fp32(w[i]) + fp32(delta[i])), i < numel.
 * Replaces add_delta_, src/blackwell_ops/cuda/lora_ops.cu:62-71 (kernel :32-38).
 */
int bw_add_delta(void* w, const void* delta, int64_t numel, void* stream);

/*
 * Fused delta + merge: w_out = add_delta(w, lora_delta(a, b, scaling)) without
 * materialising delta.  w_out may alias w (in-place merge).  fp16.
 *   w [n, k] row stride ldw; w_out [n, k] row stride ldo.
 * Composes lora_ops.cu:16-27 and :32-38; no single reference counterpart.
 */
int bw_lora_merge(const void* w, int64_t ldw, const void* a, const void* b, float scaling,
                  void* w_out, int64_t ldo, int64_t n, int64_t k, int64_t r, void* stream);

/*
 * Fused delta + merge + per-channel requantisation of the merged weight:
 * (q, scale) = quantize_weight_int8(add_delta(w, lora_delta(a, b, scaling))).
 * The merged fp16 weight is never written to memory.  q [n, k] int8 row stride
 * ldq; scale [n] fp16.  Workspace: at least bw_lora_merge_requant_workspace_size()
 * bytes (a grid-barrier count and generation, then two words per row),
 * 256-byte aligned, zero before its first use, and always passed with the same
 * workspace_bytes (its full size): each call clears the half the next call
 * uses, over that size.  After a device timeout, zero it again.  Calls sharing
 * a workspace must not overlap on the GPU.
 * Composes lora_ops.cu:16-38 and int8_gemm.py:63-68.
 */
size_t bw_lora_merge_requant_workspace_size(int64_t n, int64_t k, int64_t r);
int bw_lora_merge_requant(const void* w, int64_t ldw, const void* a, const void* b, float scaling,
                          int8_t* q, int64_t ldq, void* scale, int64_t n, int64_t k, int64_t r,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * Batched fused merge + requantisation: every problem is
 * (q, scale) = quantize_weight_int8(add_delta(w, lora_delta(a, b, scaling))),
 * e.g. all projections an adapter touches, in one launch per 16 problems
 * (problems TMA cannot address run one at a time).  Same per-problem contract
 * as bw_lora_merge_requant; one workspace of
 * bw_lora_merge_requant_batched_workspace_size() bytes serves the whole batch.
 */
typedef struct bw_lora_requant_problem {
  const void* w;   /* [n, k] fp16, row stride ldw */
  int64_t ldw;
  const void* a;   /* [r, k] fp16 contiguous */
  const void* b;   /* [n, r] fp16 contiguous */
  float scaling;
  int8_t* q;       /* [n, k] int8, row stride ldq */
  int64_t ldq;
  void* scale;     /* [n] fp16 */
  int64_t n, k, r;
} bw_lora_requant_problem;
size_t bw_lora_merge_requant_batched_workspace_size(const bw_lora_requant_problem* problems, int count);
int bw_lora_merge_requant_batched(const bw_lora_requant_problem* problems, int count, void* workspace,
                                  size_t workspace_bytes, void* stream);

/*
 * Residual + RMSNorm (the W8A16 GEMM's prologue, also callable alone).
 * Replaces fused_residual_rmsnorm / rmsnorm, src/blackwell_ops/cuda/basic_ops.cu:16-78
 * (bound at cuda/__init__.py:60-67):
 *   v = fp32(x[m,:]) + fp32(residual[m,:])   (residual == NULL: v = fp32(x[m,:]))
 *   out[m,k] = dt(v[k] * rstd * fp32(w[k])),  rstd = 1 / sqrt(sum(v^2) / K + eps)
 * with the reference kernel's summation order (256 strided partial sums, then a
 * halving tree) in IEEE fp32.  x, residual: [m, k] dtype (F16 | BF16), row stride
 * ldx; w: [k]; out: [m, k], row stride ldo.
 */
int bw_residual_rmsnorm(const void* x, const void* residual, int dtype, int64_t ldx, const void* w,
                        float eps, void* out, int64_t ldo, int64_t m, int64_t k, void* stream);

/*
 * W8A16 GEMM with the residual + RMSNorm prologue, one call:
 *   y = int8_gemm(fused_residual_rmsnorm(x, residual, norm_w, eps), w, scale)
 * (reference: basic_ops.cu:49-78 followed by int8_gemm.py:71-107).  The normalised rows are
 * written to the workspace (bw_w8a16_gemm_rmsnorm_workspace_size bytes, 256-byte aligned, the
 * first bw_w8a16_gemm_workspace_zeroed_bytes zero) and the GEMM follows with programmatic
 * dependent launch, so its weight stream overlaps the normalisation.  Results are bit-identical
 * to bw_residual_rmsnorm followed by bw_w8a16_gemm.
 */
size_t bw_w8a16_gemm_rmsnorm_workspace_size(int64_t m, int64_t n, int64_t k);
int bw_w8a16_gemm_rmsnorm(const void* x, const void* residual, int x_dtype, int64_t ldx, const void* norm_w,
                          float eps, const int8_t* w, int64_t ldw, const void* scale, int scale_dtype, void* y,
                          int64_t ldy, int64_t m, int64_t n, int64_t k, void* workspace, size_t workspace_bytes,
                          void* stream);

/*
 * Per-channel int8 quantisation of a KV-cache tensor (the quantiser family's
 * KV member).  Replaces quantize_kv_int8 / dequantize_kv_int8,
 * src/blackwell_ops/cuda/kv_quant.cu:17-58 (bound at cuda/__init__.py:78-86):
 *   x      [c, n] fp16, row stride ldx;  q [c, n] int8, row stride ldq;  scale [c] fp32
 *   scale[i] = max_j |x[i,j]| / 127 (fp32; NaN elements ignored, 0 for a row of zeros)
 *   q[i,j]   = clamp(lrint(x[i,j] / scale[i]), -127, 127)   (fp32 quotient, RNE, NaN -> 0)
 *   dequantize: x'[i,j] = fp16(fp32(q[i,j]) * scale[i])
 * Divisions are IEEE fp32.  c == 0 (or n == 0 for the dequantiser) is a no-op.
 */
int bw_quantize_kv_int8(const void* x, int64_t c, int64_t n, int64_t ldx, int8_t* q, int64_t ldq,
                        float* scale, void* stream);
int bw_dequantize_kv_int8(const int8_t* q, int64_t ldq, const float* scale, int64_t c, int64_t n,
                          void* x, int64_t ldx, void* stream);

/*
 * Device-side status of the current device: BW_OK, or BW_ERR_DEVICE_TIMEOUT
 * if a kernel's bounded wait expired since the last clear.  Synchronises
 * `stream`.  If `detail` is non-NULL it receives the failing wait site id.
 * clear != 0 resets the status to BW_OK.
 */
int bw_device_status(int clear, int* detail, void* stream);

/*
 * Bound of every spin wait inside this library's kernels (mbarrier waits, the
 * all-gather's peer-flag waits, the requantiser's grid barrier), for the
 * current device, in nanoseconds (default 4 s).  A wait that runs out records
 * its site in the device status (bw_device_status) and its kernel unwinds
 * without writing the rest of its output.  No reference counterpart: the
 * reference's kernels have no spin waits.  Takes effect for kernels launched
 * after the call; not to be changed while kernels of this library run.
 */
int bw_set_wait_limit_ns(uint64_t ns);
int bw_get_wait_limit_ns(uint64_t* ns);

/*
 * Device-side phase trace for the current device (no reference counterpart;
 * the reference profiles with torch.profiler).  While a buffer is set, each
 * CTA of a traced kernel claims one 128-byte record
 *   u64 {gridid, blockIdx | gridDim << 32, kernel id | smid << 32, t[0..12]}
 * with globaltimer stamps (ns; 0 = phase not reached).
 * Kernel ids 1 and 2, the W8A16 GEMM and its SwiGLU variant: t0 CTA start,
 * t1 first weight tile in shared memory, t2 last MMA complete, t3 epilogue
 * done, t4 the deferred stream-K reductions done, and for the all-gather
 * variant t5 the call's epoch read, t6 every peer's outputs received; t7 the
 * preceding kernel complete (griddepcontrol.wait returned).
 * Kernel id 3, the fused merge + requantisation: t0 CTA start, t1 / t4 the
 * first accumulator of pass 1 / pass 2 ready, t2 pass 1 done (grid-barrier
 * arrival), t3 grid barrier passed, t5 the last codes stored, t6 / t7 the TMA
 * producer has issued every pass-1 load / every load, t8 / t9 the first MMA
 * issuer reached pass 2 / its MMAs completed.
 * buffer = NULL turns tracing off; bw_trace_records gives the records written
 * so far (records past the buffer's capacity are dropped).
 */
int bw_trace_enable(void* buffer, size_t bytes);
int bw_trace_records(unsigned int* records);

#ifdef __cplusplus
}
#endif

#endif /* BW_OPS_H */
