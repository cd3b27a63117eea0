// Internal declarations shared by the prismaquant_b200 translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "prismaquant_b200.h"

namespace pq {

constexpr int SWEEP_THREADS = 512;
constexpr int STAGE_BYTES = 64 * 1024;     // one work item: consecutive rows, <= 64 KiB
constexpr int NSTAGE = 3;                  // shared-memory stages per CTA (192 KiB)
constexpr int MAX_ROWS_PER_ITEM = STAGE_BYTES / 32;  // cols >= 16
constexpr int FAST_STAGE_BYTES = 96 * 1024;  // fast sweep kernel: one work item
constexpr int FAST_NSTAGE = 2;                // and two stages (192 KiB)
constexpr int FAST_MAX_ROWS_PER_ITEM = 256;   // fast sweep kernel: row maxima kept in shared memory
constexpr int MAX_SWEEP_TENSORS = 320;     // descriptors per launch (kernel parameter space)

enum : int { MODE_SSE = 0, MODE_QDQ = 1 };

struct SweepDesc {
  const uint16_t* w;
  int64_t rows;
  int64_t cols;
  uint32_t fmt_mask;
  int32_t rows_per_item;
  uint8_t* nvfp4_codes;
  uint16_t* nvfp4_amax;
  uint32_t* nvfp4_tmax;
  uint16_t* out;  // QDQ output
  double* sse;    // 4 doubles (one per pq_format)
  const float* h;     // weighted sums (fast sweep, key bit 32): H per element, or per row
  int32_t h_per_row;
};

struct SweepLaunch {
  int n;
  int qdq_fmt;
  int copy_slice;      // W_hat launches: also store the weight itself, as the slice after the formats'
  int pad_;
  int64_t out_slice;   // W_hat launches: elements between format slices (0: each descriptor's rows*cols)
  int64_t item_prefix[MAX_SWEEP_TENSORS + 1];
  SweepDesc t[MAX_SWEEP_TENSORS];
};
static_assert(sizeof(SweepLaunch) <= 32764, "a SweepLaunch is passed as one kernel parameter block");

size_t sweep_smem_bytes();
size_t sweep_fast_smem_bytes();
int64_t xfmt_group(int fmt, int64_t cols);
bool mxsse_ok(const uint16_t* w, int64_t cols, int fmt);
bool intsse_ok(const uint16_t* w, int64_t cols, int fmt);
bool fp3sse_ok(const uint16_t* w, int64_t cols, int fmt);
cudaError_t launch_fp3sse(const uint16_t* w, int64_t rows, int64_t cols, double* sse, int num_sms,
                          cudaStream_t stream);
cudaError_t launch_intsse(const uint16_t* w, int64_t rows, int64_t cols, int fmt, double* sse, int num_sms,
                          cudaStream_t stream);
cudaError_t launch_mxsse(const uint16_t* w, int64_t rows, int64_t cols, const int* fmts, int nf,
                         double* const* sse, int num_sms, cudaStream_t stream);
cudaError_t launch_xfmt(const uint16_t* w, int64_t rows, int64_t cols, int fmt, double* sse, uint16_t* out,
                        int mode, int num_sms, cudaStream_t stream, const float* h = nullptr, int h_mode = 0);
cudaError_t launch_sweep_fast(const SweepLaunch& L, int grid, uint32_t key, cudaStream_t stream);
cudaError_t launch_outerr(const uint16_t* x, const uint16_t* w, const uint16_t* xq, const uint16_t* wq, int64_t batch,
                          int64_t rows, int64_t out, int64_t K, double* err_sum, double* ref_energy, float* d_ref,
                          float* d_q, cudaStream_t stream);
cudaError_t launch_outerr_ref(const uint16_t* x, const uint16_t* w, int64_t batch, int64_t rows, int64_t out,
                              int64_t K, uint16_t* y_ref, double* ref_energy, cudaStream_t stream);
cudaError_t launch_gradsq(const uint16_t* gy, const uint16_t* x, const uint16_t* w, int64_t t, int64_t m, int64_t n,
                          float* h, double* sums, cudaStream_t stream);
cudaError_t launch_outerr_err(const uint16_t* xq, const uint16_t* wq, const uint16_t* y_ref, int64_t batch,
                              int64_t rows, int64_t out, int64_t K, double* err_sum, cudaStream_t stream);
cudaError_t launch_sweep_staged(const SweepLaunch& L, int mode, int grid, cudaStream_t stream);
cudaError_t launch_sweep_generic(const uint16_t* w, int64_t rows, int64_t cols, uint32_t mask, double* sse,
                                 uint16_t* out, int mode, int num_sms, cudaStream_t stream);

// pq_pack.cu
constexpr int MAX_SCALE_SLICES = 256;
struct ScalesLaunch {
  int n;
  const uint16_t* amax[MAX_SCALE_SLICES];
  int64_t gprefix[MAX_SCALE_SLICES + 1];   // flat group offset of each slice
  uint8_t* scales[MAX_SCALE_SLICES];
  int32_t group_of[MAX_SCALE_SLICES];
  const uint32_t* tmax;
  const float* override_;
  float* global_div;
};
cudaError_t launch_nvfp4_codes(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, uint8_t* codes,
                               uint16_t* amax, uint32_t* tmax, int num_sms, cudaStream_t stream);
cudaError_t launch_nvfp4_scales(const ScalesLaunch& L, int64_t max_groups, int num_sms, cudaStream_t stream);
cudaError_t launch_nvfp4_global(const uint16_t* w, int64_t n_per, int n_slices, uint32_t* scratch, float* global_real,
                                int num_sms, cudaStream_t stream);
cudaError_t launch_mxfp8_pack(const uint16_t* w, int64_t n_elems, uint8_t* q, uint8_t* sc, int num_sms,
                              cudaStream_t stream);
cudaError_t launch_fp8_channel_pack(const uint16_t* w, int64_t rows, int64_t cols, uint8_t* q, float* scale,
                                    int num_sms, cudaStream_t stream);

// pq_fisher.cu
cudaError_t launch_sumsq_rows(const uint16_t* g, int64_t rows, int64_t cols, double* total, float* per_row,
                              int num_sms, cudaStream_t stream);
cudaError_t launch_sumsq_rows_full(const uint16_t* g, int64_t rows, int64_t cols, double* total, float* per_row,
                                   float* h, int num_sms, cudaStream_t stream);
cudaError_t launch_rownorm2(const uint16_t* x, int64_t T, int64_t d, float* out, int num_sms, cudaStream_t stream);
cudaError_t launch_tokennorm_seg(const uint16_t* g, int64_t R, int64_t d, const float* xnorm, const int64_t* tok,
                                 const int32_t* seg, double* acc, int num_sms, cudaStream_t stream);
cudaError_t launch_tokennorm_dot(const uint16_t* g, int64_t T, int64_t d, const float* xnorm,
                                 const int64_t* token_idx, double* acc, int num_sms, cudaStream_t stream);

}  // namespace pq
