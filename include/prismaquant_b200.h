/*
 * prismaquant_b200 — C ABI of the B200 (sm_100a) quantization-cost kernels.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream and returns a
 * pq_status.  Nothing here allocates or frees device memory: the caller owns
 * every input, output and scratch buffer.  bf16 tensors are passed as
 * uint16_t bit patterns, fp8 (float8_e4m3fn) and E8M0 as uint8_t.
 *
 * Paths in the comments are relative to the prismaquant project.
 */
#ifndef PRISMAQUANT_B200_H
#define PRISMAQUANT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  PQ_OK = 0,
  PQ_ERR_NULL = 1,      /* a required pointer is NULL */
  PQ_ERR_SHAPE = 2,     /* e.g. "NVFP4 group_size=16 ∤ cols" (export_native_compressed.py:1083-1084) */
  PQ_ERR_ALIGN = 3,     /* a pointer is not 16-byte aligned */
  PQ_ERR_FORMAT = 4,    /* unknown format id / empty format mask */
  PQ_ERR_CUDA = 5,      /* a CUDA launch failed (pq_last_cuda_error() has the code) */
  PQ_ERR_LIMIT = 6,     /* a size is beyond a stated maximum */
  PQ_ERR_DEVICE = 7     /* a kernel's bounded wait gave up (pq_device_error()) */
} pq_status;

/* Cost-path formats (prismaquant/format_registry.py:368-376, 418-426, 457-465, 536-546). */
typedef enum {
  PQ_FMT_NVFP4 = 0,       /* E2M1 codebook, groups of 16, real-valued amax/6 scale */
  PQ_FMT_MXFP8 = 1,       /* E4M3 codebook, groups of 32, E8M0 scale = 2^round(log2(amax/448)) */
  PQ_FMT_FP8_CHANNEL = 2, /* E4M3 codebook, one amax/448 scale per row (FP8_E4M3, group_size=0) */
  PQ_FMT_BF16 = 3,        /* passthrough: error 0 */
  PQ_NUM_FMTS = 4,        /* formats of the fused sweep (pq_sweep_sse) */
  /* The rest of the registry, served by pq_cost_qdq and pq_format_sse with exact
   * first-principles arithmetic (codebooks format_registry.py:237-300, RTN
   * :194-233, symmetric integer RTN :147-172): */
  PQ_FMT_MXFP4 = 4,          /* E2M1, groups of 32, E8M0 scale (format_registry.py:391-398) */
  PQ_FMT_MXFP6_E3M2 = 5,     /* E3M2, groups of 32, E8M0 scale (:400-407) */
  PQ_FMT_MXFP6_E2M3 = 6,     /* E2M3, groups of 32, E8M0 scale (:409-416) */
  PQ_FMT_MXFP8_E5M2 = 7,     /* E5M2, groups of 32, E8M0 scale (:436-443) */
  PQ_FMT_FP8_E5M2 = 8,       /* E5M2, one amax/cmax scale per row (:466-473) */
  PQ_FMT_NVFP3 = 9,          /* E2M0 {0, .25, .5, 1, 2}, groups of 16, real scale (:505-514) */
  PQ_FMT_INT3 = 10,          /* symmetric INT3, groups of 16 (:483-491) */
  PQ_FMT_INT2 = 11,          /* symmetric INT2, groups of 16 (:492-500) */
  PQ_FMT_INT8_CHANNEL = 12,  /* symmetric INT8, one scale per row (INT8_W8A16, :516-523) */
  PQ_FMT_INT4_G128 = 13,     /* symmetric INT4, groups of 128 (INT4_W4A16_g128, :525-533) */
  PQ_FMT_FP8_E4M3_G128 = 14, /* E4M3, groups of 128, real scale: FP8_SOURCE as the batched cost
                                path quantizes it (measure_quant_cost.py:516-548) */
  PQ_NUM_FMTS_ALL = 15
} pq_format;

#define PQ_FMT_BIT(f) (1u << (f))

/* One bf16 tensor on a sweep work list: [rows, cols] row-major, contiguous.
 * A packed-experts tensor [E, M, N] is passed as rows = E*M, cols = N.
 * fmt_mask selects formats for THIS tensor (a format whose grouping the
 * shape cannot take is left out by the caller and reported as an error
 * entry, as the reference's per-format try/except does,
 * measure_quant_cost.py:320-321, 443-444, 673-675). */
typedef struct pq_sweep_tensor {
  const uint16_t* w;
  int64_t rows;
  int64_t cols;
  uint32_t fmt_mask;
  uint32_t _pad;
  /* Optional fused NVFP4 export outputs (all three or none; needs cols % 16 == 0):
   * codes [rows, cols/2] (export_native_compressed.py:1096-1097),
   * group amax scratch [rows, cols/16] as bf16, and the tensor's running max
   * group amax as float bits (zero it before the first launch). */
  uint8_t* nvfp4_codes;
  uint16_t* nvfp4_amax;
  uint32_t* nvfp4_tmax;
} pq_sweep_tensor;

/*
 * Multi-format weight-error sweep.  For each tensor i and format f in its
 * mask, ADDS sum((W - qdq_f(W))^2) to sse[4*i + f] (fp64, device; zero it
 * first).  Replaces the per-format chain `_batched_quantize` ->
 * `err = (W - W_hat).float()` -> `err.pow(2).mean()`
 * (measure_quant_cost.py:532-548, 627-632; 411-414 for packed experts) with
 * one read of W for all formats.  weight_mse = sse / (rows*cols).
 * The reference rounds W_hat and W - W_hat to bf16 and squares in fp32;
 * so does this (an fp32 square above FLT_MAX is inf).
 * `tensors` is a HOST array; it is copied into the launch parameters.
 */
int pq_sweep_sse(const pq_sweep_tensor* tensors, int n_tensors, double* sse, void* stream);

/*
 * Cost-path quantize->dequantize of one format: w_hat = qdq_f(w) as bf16,
 * same shape.  Replaces FormatSpec.quantize_dequantize (format_registry.py:47-48,
 * 147-233) and `_batched_quantize` (measure_quant_cost.py:532-548) for every
 * format id of pq_format (0 .. PQ_NUM_FMTS_ALL - 1).
 */
int pq_cost_qdq(const uint16_t* w, int64_t rows, int64_t cols, int fmt, uint16_t* w_hat, void* stream);

/*
 * W_hat of several of the fused formats from one read of W: fmt_mask is a
 * subset of PQ_FMT_BIT(PQ_FMT_NVFP4) | PQ_FMT_BIT(PQ_FMT_MXFP8) |
 * PQ_FMT_BIT(PQ_FMT_FP8_CHANNEL), and w_hat holds popcount(fmt_mask) bf16
 * slices of rows*cols, one per format in the mask, in that order.  Each slice
 * equals pq_cost_qdq of its format.  No counterpart in the reference's API as
 * a single call; it serves measure_batched_gpu's per-format W_hat
 * (measure_quant_cost.py:628-630).
 */
int pq_cost_qdq_fused(const uint16_t* w, int64_t rows, int64_t cols, uint32_t fmt_mask, uint16_t* w_hat,
                      void* stream);

/*
 * pq_cost_qdq_fused and the error sums of the same formats from one read of a
 * stacked weight w [batch, rows, cols]: w_hat holds popcount(fmt_mask) bf16
 * slices of batch*rows*cols, one per format in the mask in format order (each
 * equal to pq_cost_qdq of its format), and sse [batch, 4] (fp64, device)
 * receives, in column f of each row b, what pq_sweep_sse would add for
 * format f of w[b].  No counterpart in the reference's API as a single call;
 * it serves measure_batched_gpu, which needs both weight_mse and W_hat of each
 * format for every Linear of a chunk (measure_quant_cost.py:628-632).
 */
int pq_cost_qdq_fused_sse(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, uint32_t fmt_mask,
                          uint16_t* w_hat, double* sse, void* stream);

/*
 * pq_cost_qdq_fused_sse for weights that are not stacked: ws holds batch device
 * pointers (a host array) to [rows, cols] bf16 weights.  w_hat holds
 * popcount(fmt_mask) + 1 slices of batch*rows*cols: the formats' W_hat as in
 * pq_cost_qdq_fused_sse, then the weights themselves stacked, written in the
 * same read (the stacked weight the other cost-table steps take).  No
 * counterpart in the reference's API as a single call; it replaces the
 * reference's torch.stack of a chunk's weights (measure_quant_cost.py:595-597)
 * together with the W_hat and weight_mse of each format.
 */
int pq_cost_qdq_fused_sse_list(const uint16_t* const* ws, int64_t batch, int64_t rows, int64_t cols,
                               uint32_t fmt_mask, uint16_t* w_hat, double* sse, void* stream);

/*
 * Sum of squared errors of one format over one bf16 tensor [rows, cols]:
 * ADDS sum((W - qdq_fmt(W))^2) (bf16 subtraction, fp32 square) to *sse
 * (fp64, device; zero it first).  fmt is one of PQ_FMT_MXFP4 ..
 * PQ_NUM_FMTS_ALL - 1, or PQ_FMT_BF16 (adds nothing); NVFP4 / MXFP8 / FP8
 * per channel go through pq_sweep_sse.  Replaces the per-format chain of
 * measure_quant_cost.py:627-632 for the formats outside the fused sweep.
 * No counterpart in the reference's API as a single call.
 */
int pq_format_sse(const uint16_t* w, int64_t rows, int64_t cols, int fmt, double* sse, void* stream);

/*
 * pq_format_sse of nf formats over one tensor: ADDS each format's sum to
 * sse[f] (fp64 device array of nf).  fmts is a HOST array of format ids, each
 * one pq_format_sse accepts; every format is checked before anything runs.
 * The MX formats among them (MXFP4, MXFP6_E3M2, MXFP6_E2M3, MXFP8_E5M2) come
 * from one read of the weights when the rows are whole 32-element groups and w
 * is 16-byte aligned.  Replaces the per-format loop of
 * measure_quant_cost.py:627-632 over those formats.
 */
int pq_format_sse_multi(const uint16_t* w, int64_t rows, int64_t cols, const int32_t* fmts, int nf, double* sse,
                        void* stream);

/*
 * H-weighted squared error of one format over one bf16 tensor [rows, cols]:
 * ADDS sum(h * (W - qdq_fmt(W))^2) to *sse (fp64, device), the square taken
 * in fp32 and then weighted.  h is fp32, one weight per element [rows, cols]
 * (h_per_row = 0) or one per row [rows] (h_per_row = 1).  Any format id
 * except that PQ_FMT_BF16 adds nothing.  predicted_dloss is half of it:
 * dense Linears with the per-weight Fisher diagonal
 * (measure_quant_cost.py:638-640), packed experts with the per-channel [E, M]
 * one, rows = E*M (:430-437, whose mean over N times N is this sum).
 */
int pq_weighted_sse(const uint16_t* w, int64_t rows, int64_t cols, int fmt, const float* h, int h_per_row,
                    double* sse, void* stream);

/*
 * pq_weighted_sse for several of the fused formats from one read of W and H:
 * fmt_mask is a subset of PQ_FMT_BIT(PQ_FMT_NVFP4) | PQ_FMT_BIT(PQ_FMT_MXFP8) |
 * PQ_FMT_BIT(PQ_FMT_FP8_CHANNEL), and sse[f] receives what pq_weighted_sse of
 * format f would add, for each f in the mask (the other entries are left
 * alone).  h as for pq_weighted_sse (16-byte aligned for the one-read path).
 * No counterpart in the reference's API as a single call; it serves
 * measure_batched_gpu's per-format predicted_dloss
 * (measure_quant_cost.py:638-640).
 */
int pq_weighted_sse_fused(const uint16_t* w, int64_t rows, int64_t cols, uint32_t fmt_mask, const float* h,
                          int h_per_row, double* sse, void* stream);

/*
 * pq_weighted_sse_fused of each w[b] of a stacked weight [batch, rows, cols]
 * with its own weights h[b] ([rows, cols], or [rows] with h_per_row = 1), in
 * one launch: sse [batch, 3] (fp64, device), row b receiving what
 * pq_weighted_sse_fused(w[b], ..., h[b], ...) would add.  No counterpart in
 * the reference's API as a single call; it serves measure_batched_gpu's
 * per-Linear predicted_dloss of a chunk (measure_quant_cost.py:638-640).
 */
int pq_weighted_sse_fused_batch(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, uint32_t fmt_mask,
                                const float* h, int h_per_row, double* sse, void* stream);

/*
 * Output error of a quantized Linear, on the tensor cores:
 *   y_ref = bf16(X W^T), y_q = bf16(X_hat W_hat^T)  (bf16 operands, fp32 accumulate)
 * ADDS sum(bf16(y_ref - y_q)^2) to err_sse[b] and sum(y_ref^2) to ref_sse[b]
 * (fp64, device; zero them first; either may be NULL) for each of `batch`
 * stacked Linears: x, x_hat are [batch, rows, k], w, w_hat [batch, out, k],
 * bf16, contiguous, 16-byte aligned, k a multiple of 8.  output_mse and
 * ref_energy are these sums over rows*out (measure_quant_cost.py:599-605,
 * 630-635, whose two bmm's and the difference this replaces, without writing
 * either product).  y_ref / y_q (fp32 [batch, rows, out], may be NULL)
 * receive the unrounded accumulators.  PQ_ERR_DEVICE if an MMA completion
 * wait gave up.
 */
int pq_output_sse(const uint16_t* x, const uint16_t* w, const uint16_t* x_hat, const uint16_t* w_hat, int64_t batch,
                  int64_t rows, int64_t out, int64_t k, double* err_sse, double* ref_sse, float* y_ref, float* y_q,
                  void* stream);

/*
 * The reference's split of the same computation (measure_quant_cost.py:599-600
 * once per chunk, :630-635 per format), each a single tensor-core GEMM:
 * pq_output_ref computes y_ref = bf16(X W^T), stores it (bf16 [batch, rows,
 * out], 16-byte aligned; may be NULL) and ADDS sum(y_ref^2) to ref_sse[b];
 * pq_output_err computes y_q = bf16(X_hat W_hat^T) and ADDS
 * sum(bf16(y_ref - y_q)^2) to err_sse[b], reading y_ref from memory.  Same
 * operand rules as pq_output_sse.
 */
/*
 * Per-weight Fisher diagonal of one backward of one Linear, on the tensor
 * cores (sensitivity_probe.py:1114-1152):
 *   grad_w = bf16(gy^T x)          gy [t, m] output gradients, x [t, n] inputs (bf16)
 *   g2 = bf16(grad_w^2);  h[m, n] += g2 (fp32, updated in place)
 *   sums[0] += sum(g2);  sums[1] += sum(bf16(g2 * bf16(w^2)))   (fp64; w [m, n] bf16, may be NULL)
 * m and n multiples of 8, pointers 16-byte aligned.  grad_w itself is never stored.
 */
int pq_grad_sq_acc(const uint16_t* gy, const uint16_t* x, const uint16_t* w, int64_t t, int64_t m, int64_t n,
                   float* h, double* sums, void* stream);

int pq_output_ref(const uint16_t* x, const uint16_t* w, int64_t batch, int64_t rows, int64_t out, int64_t k,
                  uint16_t* y_ref, double* ref_sse, void* stream);
int pq_output_err(const uint16_t* x_hat, const uint16_t* w_hat, const uint16_t* y_ref, int64_t batch, int64_t rows,
                  int64_t out, int64_t k, double* err_sse, void* stream);

/*
 * NVFP4 export, pass 1: E2M1 codes (abs-codebook RTN, ties toward zero,
 * sign from signbit; export_native_compressed.py:118-136, 226-233), the bf16
 * amax of every 16-group, and the max group amax of each of `batch`
 * consecutive [rows, cols] slices (atomic max into tmax[b], float bits;
 * zero tmax first).  Codes do not depend on the global scale
 * (export_native_compressed.py:1093-1096).
 */
int pq_nvfp4_codes(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols,
                   uint8_t* codes, uint16_t* amax, uint32_t* tmax, void* stream);

/*
 * NVFP4 export, pass 2: FP8 E4M3 block scales and the on-disk global
 * divisor for `batch` slices.  Slice b's global_real is
 *   override[b]                      if override != NULL (clamped at 1e-12),
 *   else max over slices c with group_of[c] == group_of[b] of
 *        (max_c(amax)/6)/448 clamped at 1e-12      (joint fused-sibling global,
 *        export_native_compressed.py:2090-2098; group_of == NULL: own slice)
 * scale = e4m3((amax/6 / global_real).clamp(0, 448)), global_div[b] = 1/global_real
 * (export_native_compressed.py:1045-1055, 1085-1102, 1105-1129).
 * `slices` lists `n` (amax, tmax, scale, rows*cols/16) tuples as flat arrays.
 */
int pq_nvfp4_scales(int n, const uint16_t* const* amax, const int64_t* n_groups,
                    const uint32_t* tmax_dev, const int32_t* group_of,
                    const float* override_dev, uint8_t* const* scales,
                    float* global_div_dev, void* stream);

/* compute_nvfp4_global_real (export_native_compressed.py:1045-1055) of each
 * of `batch` [rows, cols] slices from one read of the weights:
 * global_real[b] = max(max_g(max(amax_g, 1e-12) / 6) / 448, 1e-12) (IEEE
 * divisions).  scratch holds batch + 1 uint32 (zeroed here); batch <= 256. */
int pq_nvfp4_global_real(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, uint32_t* scratch,
                         float* global_real, void* stream);

/* One-call NVFP4 export of a [batch, rows, cols] tensor with a per-slice
 * global (batch == 1: quantize_dequantize_nvfp4; batch == E:
 * quantize_dequantize_nvfp4_packed, export_native_compressed.py:1058-1129).
 * override_dev may be NULL or hold `batch` floats.  scratch_amax holds
 * batch*rows*cols/16 bf16, scratch_tmax `batch` uint32 (zeroed here). */
int pq_nvfp4_pack(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols,
                  const float* override_dev, uint8_t* codes, uint8_t* scales,
                  float* global_div, uint16_t* scratch_amax, uint32_t* scratch_tmax,
                  void* stream);

/*
 * NVFP4 export for callers that cannot allocate device memory.  No
 * counterpart in the reference: it is pq_nvfp4_pack with the two scratch
 * buffers (group amax, per-slice max) replaced by a fixed array inside the
 * library, for programs whose device memory belongs to another allocator,
 * plug-in hosts that forbid device allocations, and code that must not risk
 * the device-wide synchronisation of a cudaMalloc.  The caller still passes
 * inputs and outputs; nothing is allocated or freed.
 *   Limits: batch <= 256 and batch*rows*cols/16 <= 8,388,608 groups
 *   (PQ_ERR_LIMIT otherwise).  Every GPU that loads the library holds the
 *   16 MiB + 1 KiB array until the process exits.
 *   The first call on a device looks up the array's device address with
 *   cudaGetSymbolAddress (that device current); make it before any stream
 *   capture.  The address is kept for the process's lifetime, so the entry
 *   point must not be used on a device after a cudaDeviceReset of it.  All
 *   calls on a device share the array: calls that overlap on the GPU race;
 *   each call clears the per-slice maxima it uses.  It runs the same codes
 *   and scales passes as pq_nvfp4_pack, so bytes and speed are the same.
 */
int pq_nvfp4_pack_noalloc(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols,
                          const float* override_dev, uint8_t* codes, uint8_t* scales, float* global_div,
                          void* stream);

/*
 * MXFP8 export (quantize_dequantize_mxfp8[_packed], export_native_compressed.py:1135-1194):
 * E8M0 exponent e = clamp(ceil(log2(max(amax32, 2^-127)/448)), -127, 127)
 * (torch float32 log2 semantics), q = e4m3((w / 2^e).clamp(+-448)),
 * scale byte = e + 127.  n_rows*cols elements, cols % 32 == 0.
 */
int pq_mxfp8_pack(const uint16_t* w, int64_t n_rows, int64_t cols, uint8_t* q, uint8_t* scale_e8m0,
                  void* stream);

/*
 * FP8 per-channel export (quantize_dequantize_fp8_dynamic[_packed],
 * export_native_compressed.py:1197-1226): s = max(row amax, 2^-127)/448,
 * q = e4m3((w / s).clamp(+-448)); scale [n_rows] fp32.
 */
int pq_fp8_channel_pack(const uint16_t* w, int64_t n_rows, int64_t cols, uint8_t* q, float* scale,
                        void* stream);

/*
 * Fisher statistics.
 *
 * pq_sumsq_rows: _GradNormCapture.backward (sensitivity_probe.py:451-482):
 * total += sum(g^2) (fp64, device scalar) and, if per_row != NULL,
 * per_row[r] += sum_n g[r, n]^2 (fp32; the [E, M] channel diagonal).
 */
int pq_sumsq_rows(const uint16_t* g, int64_t n_rows, int64_t cols, double* total, float* per_row,
                  void* stream);

/* pq_sumsq_rows_full: pq_sumsq_rows plus the per-weight accumulator of
 * _GradNormCapture's full_accumulator (sensitivity_probe.py:486-503):
 * h_full[i] += fp32(g[i])^2 (fp32, one IEEE add per element, bit-exact with the
 * reference's `cur.add_(g.float().pow(2))`), from the same read of g.
 * h_full has n_rows*cols floats. */
int pq_sumsq_rows_full(const uint16_t* g, int64_t n_rows, int64_t cols, double* total, float* per_row,
                       float* h_full, void* stream);

/* pq_rownorm2: out[t] = sum_d x[t, d]^2 (fp32) for x [T, d] bf16 — the
 * forward half of the per-token estimator that replaces the
 * GEMM-then-square in FisherAccumulator._make_bwd (sensitivity_probe.py:1115-1152). */
int pq_rownorm2(const uint16_t* x, int64_t T, int64_t d, float* out, void* stream);

/* pq_tokennorm_dot: acc[0] += sum_t xnorm[idx(t)] * sum_d g[t, d]^2 (fp64),
 * idx(t) = token_idx ? token_idx[t] : t.  With token_idx it serves the
 * routed (per-expert) estimator for packed experts; acc[1] += T (tokens). */
int pq_tokennorm_dot(const uint16_t* g, int64_t T, int64_t d, const float* xnorm,
                     const int64_t* token_idx, double* acc, void* stream);

/* Housekeeping. */
/* pq_tokennorm_dot_seg: the per-token Fisher estimate of a routed packed-expert
 * projection in one launch (north-star form of sensitivity_probe.py:555-728's
 * per-expert loop).  g [R, d] bf16 holds the output gradients of the R (token,
 * expert) rows, sorted by expert; seg[r] in [0, n_seg) is row r's expert and
 * token_idx[r] its token (NULL: xnorm is already per row).  For each expert e:
 * acc[2e] += sum_{r in e} xnorm[token(r)] * ||g_r||^2, acc[2e+1] += its rows.
 * Rows of one expert must be contiguous. */
int pq_tokennorm_dot_seg(const uint16_t* g, int64_t R, int64_t d, const float* xnorm, const int64_t* token_idx,
                         const int32_t* seg, int64_t n_seg, double* acc, void* stream);

int pq_device_error(int* code);          /* reads and clears the device error word */

/* Failure-detection hook (no counterpart in the reference): the iteration
 * limit of the sweep kernels' waits for a work item's bulk copy, on the
 * current device.  A kernel whose wait runs out records ERR_MBAR_TIMEOUT (1)
 * in the device error word, waits with a fixed limit for the copies it has
 * issued, and returns; pq_device_error() then reports it.  0 makes every such
 * wait give up at once (tests); pq_default_wait_limit() restores the default.
 * Synchronous with respect to the host; not for use while sweeps are running. */
int pq_set_wait_limit(uint32_t iterations);
uint32_t pq_default_wait_limit(void);
int pq_last_cuda_error(void);
const char* pq_status_string(int status);
int pq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PRISMAQUANT_B200_H */
