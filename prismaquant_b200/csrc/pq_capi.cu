// C ABI entry points (include/prismaquant_b200.h): argument validation, path
// selection and launch batching around the kernels.  No entry point allocates
// device memory or synchronizes the stream.
#include <atomic>
#include <string.h>

#include <vector>

#include "pq_common.cuh"
#include "pq_internal.h"

namespace {

thread_local int t_last_cuda_error = 0;

int num_sms_current() {
  static std::atomic<int> cached[64];   // per device; host threads may race to fill a slot with one value
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  int v = cached[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cached[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

inline int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return PQ_OK;
  t_last_cuda_error = (int)e;
  return PQ_ERR_CUDA;
}

constexpr uint32_t NV = PQ_FMT_BIT(PQ_FMT_NVFP4);
constexpr uint32_t MX = PQ_FMT_BIT(PQ_FMT_MXFP8);
constexpr uint32_t F8 = PQ_FMT_BIT(PQ_FMT_FP8_CHANNEL);
constexpr uint32_t ALL_FMTS = 0xFu;

// Shape rules of the reference's grouping (format_registry.py:208-212): a
// group longer than the row becomes the whole row; otherwise the row must
// divide into groups.
int check_groups(int64_t cols, uint32_t mask) {
  if ((mask & NV) && cols > 16 && cols % 16) return PQ_ERR_SHAPE;
  if ((mask & MX) && cols > 32 && cols % 32) return PQ_ERR_SHAPE;
  return PQ_OK;
}

bool staged_ok(const uint16_t* w, int64_t cols, uint32_t mask) {
  if (cols % 16 || cols < 16 || cols * 2 > pq::STAGE_BYTES || !aligned(w, 16)) return false;
  if ((mask & MX) && cols % 32) return false;
  return true;
}

// out_slice: W_hat launches, elements between format slices (0: each descriptor's rows*cols).
// copy_slice: W_hat launches, also store each weight as the slice after the formats.
int launch_batch(std::vector<pq::SweepDesc>& descs, int mode, int qfmt, uint32_t key, cudaStream_t stream,
                 int64_t out_slice = 0, int copy_slice = 0) {
  size_t i = 0;
  const int sms = num_sms_current();
  while (i < descs.size()) {
    pq::SweepLaunch L;
    memset(&L, 0, sizeof(L));
    L.qdq_fmt = qfmt;
    L.out_slice = out_slice;
    L.copy_slice = copy_slice;
    int64_t items = 0;
    int n = 0;
    for (; i < descs.size() && n < pq::MAX_SWEEP_TENSORS; ++i, ++n) {
      pq::SweepDesc d = descs[i];
      int64_t rpi = (mode == pq::MODE_SSE ? pq::FAST_STAGE_BYTES : pq::STAGE_BYTES) / (d.cols * 2);
      if (mode == pq::MODE_SSE && rpi > pq::FAST_MAX_ROWS_PER_ITEM) rpi = pq::FAST_MAX_ROWS_PER_ITEM;
      if (rpi > d.rows) rpi = d.rows;
      if (rpi < 1) rpi = 1;
      d.rows_per_item = (int32_t)rpi;
      L.t[n] = d;
      L.item_prefix[n] = items;
      items += (d.rows + rpi - 1) / rpi;
    }
    L.n = n;
    L.item_prefix[n] = items;
    if (items == 0) continue;
    const int grid = (int)(items < sms ? items : sms);
    const int st = cuda_status(mode == pq::MODE_SSE ? pq::launch_sweep_fast(L, grid, key, stream)
                                                    : pq::launch_sweep_staged(L, mode, grid, stream));
    if (st) return st;
  }
  return PQ_OK;
}

// Launch the staged descriptors; the fast sweep kernel is specialised on the
// format set, so descriptors are grouped by (format mask, NVFP4 codes).
int flush_staged(std::vector<pq::SweepDesc>& descs, int mode, int qfmt, cudaStream_t stream) {
  if (mode != pq::MODE_SSE) {
    const int st = launch_batch(descs, mode, qfmt, 0u, stream);
    descs.clear();
    return st;
  }
  for (uint32_t key = 1; key < 16; ++key) {
    std::vector<pq::SweepDesc> group;
    for (const auto& d : descs)
      if (((d.fmt_mask & 7u) | (d.nvfp4_codes ? 8u : 0u)) == key) group.push_back(d);
    if (group.empty()) continue;
    const int st = launch_batch(group, mode, qfmt, key, stream);
    if (st) return st;
  }
  descs.clear();
  return PQ_OK;
}

}  // namespace

extern "C" {

int pq_version(void) { return 1; }

int pq_last_cuda_error(void) { return t_last_cuda_error; }

const char* pq_status_string(int s) {
  switch (s) {
    case PQ_OK: return "ok";
    case PQ_ERR_NULL: return "null pointer";
    case PQ_ERR_SHAPE: return "shape not divisible by the format's group size";
    case PQ_ERR_ALIGN: return "pointer not aligned as required";
    case PQ_ERR_FORMAT: return "unknown format";
    case PQ_ERR_CUDA: return "CUDA launch error";
    case PQ_ERR_LIMIT: return "size beyond the supported maximum";
    case PQ_ERR_DEVICE: return "a kernel's bounded wait gave up";
    default: return "unknown status";
  }
}

int pq_device_error(int* code) {
  if (!code) return PQ_ERR_NULL;
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, pq::g_pq_device_error, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e);
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(pq::g_pq_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e);
  }
  *code = v;
  return PQ_OK;
}

int pq_set_wait_limit(uint32_t iterations) {
  return cuda_status(cudaMemcpyToSymbol(pq::g_pq_wait_limit, &iterations, sizeof(uint32_t)));
}

uint32_t pq_default_wait_limit(void) { return pq::DEFAULT_WAIT_LIMIT; }

int pq_sweep_sse(const pq_sweep_tensor* ts, int n, double* sse, void* stream_) {
  if (n < 0) return PQ_ERR_SHAPE;
  if (n == 0) return PQ_OK;
  if (!ts || !sse) return PQ_ERR_NULL;
  cudaStream_t stream = (cudaStream_t)stream_;
  std::vector<pq::SweepDesc> staged;
  // validate everything before launching anything
  for (int i = 0; i < n; ++i) {
    const pq_sweep_tensor& t = ts[i];
    if (t.rows < 0 || t.cols < 1) return PQ_ERR_SHAPE;
    if (t.fmt_mask & ~ALL_FMTS) return PQ_ERR_FORMAT;
    if (t.rows > 0 && !t.w) return PQ_ERR_NULL;
    const int st = check_groups(t.cols, t.fmt_mask);
    if (st) return st;
    const bool codes = t.nvfp4_codes || t.nvfp4_amax || t.nvfp4_tmax;
    if (codes) {
      if (!t.nvfp4_codes || !t.nvfp4_amax || !t.nvfp4_tmax) return PQ_ERR_NULL;
      if (t.cols % 16) return PQ_ERR_SHAPE;
      if (!aligned(t.w, 16) || !aligned(t.nvfp4_codes, 4) || !aligned(t.nvfp4_amax, 2) || !aligned(t.nvfp4_tmax, 4))
        return PQ_ERR_ALIGN;
    }
  }
  const int sms = num_sms_current();
  for (int i = 0; i < n; ++i) {
    const pq_sweep_tensor& t = ts[i];
    const uint32_t m = t.fmt_mask & (NV | MX | F8);
    const bool codes = t.nvfp4_codes != nullptr;
    if (t.rows == 0) continue;
    if (staged_ok(t.w, t.cols, m)) {
      pq::SweepDesc d;
      memset(&d, 0, sizeof(d));
      d.w = t.w;
      d.rows = t.rows;
      d.cols = t.cols;
      d.fmt_mask = m;
      d.sse = sse + 4 * (int64_t)i;
      if (codes) {
        d.nvfp4_codes = t.nvfp4_codes;
        d.nvfp4_amax = t.nvfp4_amax;
        d.nvfp4_tmax = t.nvfp4_tmax;
      }
      if (m || codes) staged.push_back(d);
    } else {
      if (m) {
        const int st = cuda_status(pq::launch_sweep_generic(t.w, t.rows, t.cols, m, sse + 4 * (int64_t)i, nullptr,
                                                            pq::MODE_SSE, sms, stream));
        if (st) return st;
      }
      if (codes) {
        const int st = cuda_status(pq::launch_nvfp4_codes(t.w, 1, t.rows, t.cols, t.nvfp4_codes, t.nvfp4_amax,
                                                          t.nvfp4_tmax, sms, stream));
        if (st) return st;
      }
    }
  }
  return flush_staged(staged, pq::MODE_SSE, 0, stream);
}

int pq_format_sse(const uint16_t* w, int64_t rows, int64_t cols, int fmt, double* sse, void* stream_) {
  if (rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (fmt != PQ_FMT_BF16 && !pq::xfmt_known(fmt)) return PQ_ERR_FORMAT;
  if (fmt != PQ_FMT_BF16 && pq::xfmt_group(fmt, cols) == 0) return PQ_ERR_SHAPE;
  if (rows == 0 || fmt == PQ_FMT_BF16) return PQ_OK;
  if (!w || !sse) return PQ_ERR_NULL;
  if (pq::mxsse_ok(w, cols, fmt))
    return cuda_status(pq::launch_mxsse(w, rows, cols, &fmt, 1, &sse, num_sms_current(), (cudaStream_t)stream_));
  if (pq::intsse_ok(w, cols, fmt))
    return cuda_status(pq::launch_intsse(w, rows, cols, fmt, sse, num_sms_current(), (cudaStream_t)stream_));
  if (pq::fp3sse_ok(w, cols, fmt))
    return cuda_status(pq::launch_fp3sse(w, rows, cols, sse, num_sms_current(), (cudaStream_t)stream_));
  return cuda_status(pq::launch_xfmt(w, rows, cols, fmt, sse, nullptr, pq::MODE_SSE, num_sms_current(),
                                     (cudaStream_t)stream_));
}

int pq_format_sse_multi(const uint16_t* w, int64_t rows, int64_t cols, const int32_t* fmts, int nf, double* sse,
                        void* stream_) {
  if (nf < 0 || (nf > 0 && !fmts)) return PQ_ERR_NULL;
  if (rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  for (int f = 0; f < nf; ++f) {   // every format checked before anything runs
    if (fmts[f] != PQ_FMT_BF16 && !pq::xfmt_known(fmts[f])) return PQ_ERR_FORMAT;
    if (fmts[f] != PQ_FMT_BF16 && pq::xfmt_group(fmts[f], cols) == 0) return PQ_ERR_SHAPE;
  }
  if (rows == 0 || nf == 0) return PQ_OK;
  if (!w || !sse) return PQ_ERR_NULL;
  const cudaStream_t stream = (cudaStream_t)stream_;
  const int sms = num_sms_current();
  int mx[8];
  double* mx_sse[8];
  int n_mx = 0;
  for (int f = 0; f < nf; ++f) {
    if (fmts[f] == PQ_FMT_BF16) continue;
    const int fmt = fmts[f];
    bool seen = false;   // a repeated MX format goes on its own
    for (int i = 0; i < n_mx; ++i) seen = seen || mx[i] == fmt;
    if (!seen && n_mx < 8 && pq::mxsse_ok(w, cols, fmt)) {   // the MX formats from one read
      mx[n_mx] = fmt;
      mx_sse[n_mx++] = sse + f;
      continue;
    }
    if (pq::mxsse_ok(w, cols, fmt)) {
      double* one = sse + f;
      const int st = cuda_status(pq::launch_mxsse(w, rows, cols, &fmt, 1, &one, sms, stream));
      if (st != PQ_OK) return st;
      continue;
    }
    const int st = pq::intsse_ok(w, cols, fmt)
                       ? cuda_status(pq::launch_intsse(w, rows, cols, fmt, sse + f, sms, stream))
                   : pq::fp3sse_ok(w, cols, fmt)
                       ? cuda_status(pq::launch_fp3sse(w, rows, cols, sse + f, sms, stream))
                       : cuda_status(pq::launch_xfmt(w, rows, cols, fmt, sse + f, nullptr, pq::MODE_SSE, sms, stream));
    if (st != PQ_OK) return st;
  }
  if (n_mx > 0) return cuda_status(pq::launch_mxsse(w, rows, cols, mx, n_mx, mx_sse, sms, stream));
  return PQ_OK;
}

int pq_weighted_sse(const uint16_t* w, int64_t rows, int64_t cols, int fmt, const float* h, int h_per_row,
                    double* sse, void* stream_) {
  if (rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (fmt != PQ_FMT_BF16 && !pq::xfmt_scorable(fmt)) return PQ_ERR_FORMAT;
  if (fmt != PQ_FMT_BF16 && pq::xfmt_group(fmt, cols) == 0) return PQ_ERR_SHAPE;
  if (rows == 0 || fmt == PQ_FMT_BF16) return PQ_OK;
  if (!w || !h || !sse) return PQ_ERR_NULL;
  return cuda_status(pq::launch_xfmt(w, rows, cols, fmt, sse, nullptr, pq::MODE_SSE, num_sms_current(),
                                     (cudaStream_t)stream_, h, h_per_row ? 2 : 1));
}

int pq_weighted_sse_fused(const uint16_t* w, int64_t rows, int64_t cols, uint32_t fmt_mask, const float* h,
                          int h_per_row, double* sse, void* stream_) {
  if (rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (fmt_mask == 0 || (fmt_mask & ~(NV | MX | F8))) return PQ_ERR_FORMAT;
  const int st0 = check_groups(cols, fmt_mask);
  if (st0) return st0;
  if (rows == 0) return PQ_OK;
  if (!w || !h || !sse) return PQ_ERR_NULL;
  if (staged_ok(w, cols, fmt_mask) && (h_per_row || aligned(h, 16))) {   // one read of W and H
    std::vector<pq::SweepDesc> v(1);
    memset(&v[0], 0, sizeof(pq::SweepDesc));
    v[0].w = w;
    v[0].rows = rows;
    v[0].cols = cols;
    v[0].fmt_mask = fmt_mask;
    v[0].sse = sse;
    v[0].h = h;
    v[0].h_per_row = h_per_row ? 1 : 0;
    return launch_batch(v, pq::MODE_SSE, 0, fmt_mask | 32u, (cudaStream_t)stream_);
  }
  for (int f = 0; f < 3; ++f) {   // other shapes: one format at a time
    if (!(fmt_mask & (1u << f))) continue;
    const int st = pq_weighted_sse(w, rows, cols, f, h, h_per_row, sse + f, stream_);
    if (st) return st;
  }
  return PQ_OK;
}

int pq_weighted_sse_fused_batch(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, uint32_t fmt_mask,
                                const float* h, int h_per_row, double* sse, void* stream_) {
  if (batch < 0 || rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (fmt_mask == 0 || (fmt_mask & ~(NV | MX | F8))) return PQ_ERR_FORMAT;
  const int st0 = check_groups(cols, fmt_mask);
  if (st0) return st0;
  if (batch == 0 || rows == 0) return PQ_OK;
  if (!w || !h || !sse) return PQ_ERR_NULL;
  const int64_t per = rows * cols, hper = h_per_row ? rows : per;
  if (staged_ok(w, cols, fmt_mask) && (h_per_row || aligned(h, 16))) {   // one launch for the batch
    std::vector<pq::SweepDesc> v((size_t)batch);
    for (int64_t b = 0; b < batch; ++b) {
      memset(&v[b], 0, sizeof(pq::SweepDesc));
      v[b].w = w + b * per;
      v[b].rows = rows;
      v[b].cols = cols;
      v[b].fmt_mask = fmt_mask;
      v[b].sse = sse + 3 * b;
      v[b].h = h + b * hper;
      v[b].h_per_row = h_per_row ? 1 : 0;
    }
    return launch_batch(v, pq::MODE_SSE, 0, fmt_mask | 32u, (cudaStream_t)stream_);
  }
  for (int64_t b = 0; b < batch; ++b) {   // other shapes: one tensor at a time
    const int st = pq_weighted_sse_fused(w + b * per, rows, cols, fmt_mask, h + b * hper, h_per_row, sse + 3 * b,
                                         stream_);
    if (st) return st;
  }
  return PQ_OK;
}

// Shapes the output-error kernels take: k % 8 == 0 (16-byte tensor-map strides), grid limits.
static int outerr_shape(int64_t batch, int64_t rows, int64_t out, int64_t k) {
  if (batch < 0 || rows < 0 || out < 0 || k < 1 || (k & 7)) return PQ_ERR_SHAPE;
  if (batch > 65535 || (rows + 127) / 128 > 0x7fffffff || (out + 127) / 128 > 65535 || k > (int64_t)1 << 31)
    return PQ_ERR_LIMIT;
  return PQ_OK;
}

int pq_cost_qdq_fused(const uint16_t* w, int64_t rows, int64_t cols, uint32_t fmt_mask, uint16_t* w_hat,
                      void* stream_) {
  if (rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  const uint32_t fused = NV | MX | F8;
  if (fmt_mask == 0 || (fmt_mask & ~fused)) return PQ_ERR_FORMAT;
  const int st0 = check_groups(cols, fmt_mask);
  if (st0) return st0;
  if (rows == 0) return PQ_OK;
  if (!w || !w_hat) return PQ_ERR_NULL;
  if (staged_ok(w, cols, fmt_mask) && aligned(w_hat, 16)) {   // one read of W for every format
    std::vector<pq::SweepDesc> v(1);
    memset(&v[0], 0, sizeof(pq::SweepDesc));
    v[0].w = w;
    v[0].rows = rows;
    v[0].cols = cols;
    v[0].fmt_mask = fmt_mask;
    v[0].out = w_hat;
    return launch_batch(v, pq::MODE_SSE, 0, fmt_mask | 16u, (cudaStream_t)stream_);
  }
  int slot = 0;   // other shapes: one W_hat at a time, same slices
  for (int f = 0; f < 3; ++f) {
    if (!(fmt_mask & (1u << f))) continue;
    const int st = pq_cost_qdq(w, rows, cols, f, w_hat + (int64_t)slot * rows * cols, stream_);
    if (st) return st;
    ++slot;
  }
  return PQ_OK;
}

int pq_cost_qdq_fused_sse(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, uint32_t fmt_mask,
                          uint16_t* w_hat, double* sse, void* stream_) {
  if (batch < 0 || rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (fmt_mask == 0 || (fmt_mask & ~(NV | MX | F8))) return PQ_ERR_FORMAT;
  const int st0 = check_groups(cols, fmt_mask);
  if (st0) return st0;
  if (batch == 0 || rows == 0) return PQ_OK;
  if (!w || !w_hat || !sse) return PQ_ERR_NULL;
  if (batch > 0x7fffffff) return PQ_ERR_LIMIT;
  const int64_t per = rows * cols;
  cudaStream_t stream = (cudaStream_t)stream_;
  if (staged_ok(w, cols, fmt_mask) && aligned(w_hat, 16)) {   // one read of W: W_hat and the sums
    std::vector<pq::SweepDesc> v((size_t)batch);
    for (int64_t b = 0; b < batch; ++b) {
      memset(&v[b], 0, sizeof(pq::SweepDesc));
      v[b].w = w + b * per;
      v[b].rows = rows;
      v[b].cols = cols;
      v[b].fmt_mask = fmt_mask;
      v[b].out = w_hat + b * per;
      v[b].sse = sse + 4 * b;
    }
    return launch_batch(v, pq::MODE_SSE, 0, fmt_mask | 16u | 64u, stream, batch * per);
  }
  // other shapes: the W_hat slices as pq_cost_qdq_fused writes them, the sums as pq_sweep_sse adds them
  const int st = pq_cost_qdq_fused(w, batch * rows, cols, fmt_mask, w_hat, stream_);
  if (st) return st;
  std::vector<pq_sweep_tensor> ts((size_t)batch);
  for (int64_t b = 0; b < batch; ++b) {
    memset(&ts[b], 0, sizeof(pq_sweep_tensor));
    ts[b].w = w + b * per;
    ts[b].rows = rows;
    ts[b].cols = cols;
    ts[b].fmt_mask = fmt_mask;
  }
  return pq_sweep_sse(ts.data(), (int)batch, sse, stream_);
}

int pq_cost_qdq_fused_sse_list(const uint16_t* const* ws, int64_t batch, int64_t rows, int64_t cols,
                               uint32_t fmt_mask, uint16_t* w_hat, double* sse, void* stream_) {
  if (batch < 0 || rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (fmt_mask == 0 || (fmt_mask & ~(NV | MX | F8))) return PQ_ERR_FORMAT;
  const int st0 = check_groups(cols, fmt_mask);
  if (st0) return st0;
  if (batch == 0 || rows == 0) return PQ_OK;
  if (!ws || !w_hat || !sse) return PQ_ERR_NULL;
  if (batch > 0x7fffffff) return PQ_ERR_LIMIT;
  bool staged = aligned(w_hat, 16);
  for (int64_t b = 0; b < batch; ++b) {
    if (!ws[b]) return PQ_ERR_NULL;
    staged = staged && staged_ok(ws[b], cols, fmt_mask);
  }
  const int64_t per = rows * cols;
  const int nf = __builtin_popcount(fmt_mask);
  uint16_t* copy = w_hat + (int64_t)nf * batch * per;   // the stacked weight, after the format slices
  cudaStream_t stream = (cudaStream_t)stream_;
  if (staged) {   // one read of each weight: W_hat, the sums and the stacked copy
    std::vector<pq::SweepDesc> v((size_t)batch);
    for (int64_t b = 0; b < batch; ++b) {
      memset(&v[b], 0, sizeof(pq::SweepDesc));
      v[b].w = ws[b];
      v[b].rows = rows;
      v[b].cols = cols;
      v[b].fmt_mask = fmt_mask;
      v[b].out = w_hat + b * per;
      v[b].sse = sse + 4 * b;
    }
    return launch_batch(v, pq::MODE_SSE, 0, fmt_mask | 16u | 64u, stream, batch * per, 1);
  }
  // other shapes or alignments: stack the weights into the copy slice, then work on the copy
  for (int64_t b = 0; b < batch; ++b) {
    const int st = cuda_status(cudaMemcpyAsync(copy + b * per, ws[b], (size_t)per * 2, cudaMemcpyDeviceToDevice,
                                               stream));
    if (st) return st;
  }
  return pq_cost_qdq_fused_sse(copy, batch, rows, cols, fmt_mask, w_hat, sse, stream_);
}

int pq_grad_sq_acc(const uint16_t* gy, const uint16_t* x, const uint16_t* w, int64_t t, int64_t m, int64_t n,
                   float* h, double* sums, void* stream_) {
  if (t < 0 || m < 0 || n < 0 || (m & 7) || (n & 7)) return PQ_ERR_SHAPE;
  if (t > 0x7fffffff || (m + 255) / 256 > 0x3fffffff || (n + 255) / 256 > 65535) return PQ_ERR_LIMIT;
  if (t == 0 || m == 0 || n == 0) return PQ_OK;
  if (!gy || !x || !h || !sums) return PQ_ERR_NULL;
  if (!aligned(gy, 16) || !aligned(x, 16) || !aligned(h, 16) || !aligned(w, 16)) return PQ_ERR_ALIGN;
  return cuda_status(pq::launch_gradsq(gy, x, w, t, m, n, h, sums, (cudaStream_t)stream_));
}

int pq_output_sse(const uint16_t* x, const uint16_t* w, const uint16_t* x_hat, const uint16_t* w_hat, int64_t batch,
                  int64_t rows, int64_t out, int64_t k, double* err_sse, double* ref_sse, float* y_ref, float* y_q,
                  void* stream_) {
  const int st = outerr_shape(batch, rows, out, k);
  if (st) return st;
  if (batch == 0 || rows == 0 || out == 0) return PQ_OK;
  if (!x || !w || !x_hat || !w_hat) return PQ_ERR_NULL;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(x_hat, 16) || !aligned(w_hat, 16)) return PQ_ERR_ALIGN;
  return cuda_status(pq::launch_outerr(x, w, x_hat, w_hat, batch, rows, out, k, err_sse, ref_sse, y_ref, y_q,
                                       (cudaStream_t)stream_));
}

int pq_output_ref(const uint16_t* x, const uint16_t* w, int64_t batch, int64_t rows, int64_t out, int64_t k,
                  uint16_t* y_ref, double* ref_sse, void* stream_) {
  const int st = outerr_shape(batch, rows, out, k);
  if (st) return st;
  if (batch == 0 || rows == 0 || out == 0) return PQ_OK;
  if (!x || !w) return PQ_ERR_NULL;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y_ref, 16)) return PQ_ERR_ALIGN;
  return cuda_status(pq::launch_outerr_ref(x, w, batch, rows, out, k, y_ref, ref_sse, (cudaStream_t)stream_));
}

int pq_output_err(const uint16_t* x_hat, const uint16_t* w_hat, const uint16_t* y_ref, int64_t batch, int64_t rows,
                  int64_t out, int64_t k, double* err_sse, void* stream_) {
  const int st = outerr_shape(batch, rows, out, k);
  if (st) return st;
  if (batch == 0 || rows == 0 || out == 0) return PQ_OK;
  if (!x_hat || !w_hat || !y_ref) return PQ_ERR_NULL;
  if (!aligned(x_hat, 16) || !aligned(w_hat, 16) || !aligned(y_ref, 16)) return PQ_ERR_ALIGN;
  return cuda_status(pq::launch_outerr_err(x_hat, w_hat, y_ref, batch, rows, out, k, err_sse, (cudaStream_t)stream_));
}

int pq_cost_qdq(const uint16_t* w, int64_t rows, int64_t cols, int fmt, uint16_t* w_hat, void* stream_) {
  if (rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (fmt < 0 || fmt >= PQ_NUM_FMTS_ALL) return PQ_ERR_FORMAT;
  if (pq::xfmt_known(fmt)) {
    if (pq::xfmt_group(fmt, cols) == 0) return PQ_ERR_SHAPE;
    if (rows == 0) return PQ_OK;
    if (!w || !w_hat) return PQ_ERR_NULL;
    return cuda_status(pq::launch_xfmt(w, rows, cols, fmt, nullptr, w_hat, pq::MODE_QDQ, num_sms_current(),
                                       (cudaStream_t)stream_));
  }
  if (rows == 0) return PQ_OK;
  if (!w || !w_hat) return PQ_ERR_NULL;
  cudaStream_t stream = (cudaStream_t)stream_;
  if (fmt == PQ_FMT_BF16)
    return cuda_status(cudaMemcpyAsync(w_hat, w, (size_t)rows * cols * 2, cudaMemcpyDeviceToDevice, stream));
  const uint32_t m = 1u << fmt;
  const int st = check_groups(cols, m);
  if (st) return st;
  if (staged_ok(w, cols, m) && aligned(w_hat, 16)) {   // the fast sweep kernel's W_hat mode
    std::vector<pq::SweepDesc> v(1);
    memset(&v[0], 0, sizeof(pq::SweepDesc));
    v[0].w = w;
    v[0].rows = rows;
    v[0].cols = cols;
    v[0].fmt_mask = m;
    v[0].out = w_hat;
    return launch_batch(v, pq::MODE_SSE, 0, m | 16u, stream);
  }
  return cuda_status(pq::launch_sweep_generic(w, rows, cols, m, nullptr, w_hat, pq::MODE_QDQ, num_sms_current(),
                                              stream));
}

int pq_nvfp4_codes(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, uint8_t* codes, uint16_t* amax,
                   uint32_t* tmax, void* stream) {
  if (batch < 0 || rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (cols % 16) return PQ_ERR_SHAPE;
  if (batch == 0 || rows == 0) return PQ_OK;
  if (!w || !codes || !amax || !tmax) return PQ_ERR_NULL;
  if (!aligned(w, 16) || !aligned(codes, 4) || !aligned(amax, 2) || !aligned(tmax, 4)) return PQ_ERR_ALIGN;
  if (staged_ok(w, cols, NV) && aligned(codes, 8)) {
    // the fast sweep kernel's codes-only form (the fused export's pass 1), one descriptor per slice
    std::vector<pq::SweepDesc> v((size_t)batch);
    for (int64_t b = 0; b < batch; ++b) {
      memset(&v[b], 0, sizeof(pq::SweepDesc));
      v[b].w = w + b * rows * cols;
      v[b].rows = rows;
      v[b].cols = cols;
      v[b].nvfp4_codes = codes + b * rows * cols / 2;
      v[b].nvfp4_amax = amax + b * rows * cols / 16;
      v[b].nvfp4_tmax = tmax + b;
    }
    return launch_batch(v, pq::MODE_SSE, 0, 8u, (cudaStream_t)stream);
  }
  return cuda_status(
      pq::launch_nvfp4_codes(w, batch, rows, cols, codes, amax, tmax, num_sms_current(), (cudaStream_t)stream));
}

int pq_nvfp4_scales(int n, const uint16_t* const* amax, const int64_t* n_groups, const uint32_t* tmax_dev,
                    const int32_t* group_of, const float* override_dev, uint8_t* const* scales,
                    float* global_div_dev, void* stream) {
  if (n < 0) return PQ_ERR_SHAPE;
  if (n == 0) return PQ_OK;
  if (n > pq::MAX_SCALE_SLICES) return PQ_ERR_LIMIT;
  if (!amax || !n_groups || !scales || !global_div_dev || (!tmax_dev && !override_dev)) return PQ_ERR_NULL;
  pq::ScalesLaunch L;
  memset(&L, 0, sizeof(L));
  L.n = n;
  int64_t maxg = 0;
  L.gprefix[0] = 0;
  for (int i = 0; i < n; ++i) {
    if (n_groups[i] < 0) return PQ_ERR_SHAPE;
    if (n_groups[i] > 0 && (!amax[i] || !scales[i])) return PQ_ERR_NULL;
    L.amax[i] = amax[i];
    L.gprefix[i + 1] = L.gprefix[i] + n_groups[i];
    L.scales[i] = scales[i];
    L.group_of[i] = group_of ? group_of[i] : -1;
    if (n_groups[i] > maxg) maxg = n_groups[i];
  }
  L.tmax = tmax_dev;
  L.override_ = override_dev;
  L.global_div = global_div_dev;
  return cuda_status(pq::launch_nvfp4_scales(L, maxg, num_sms_current(), (cudaStream_t)stream));
}

int pq_nvfp4_pack(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, const float* override_dev,
                  uint8_t* codes, uint8_t* scales, float* global_div, uint16_t* scratch_amax,
                  uint32_t* scratch_tmax, void* stream_) {
  if (batch < 0 || rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (cols % 16) return PQ_ERR_SHAPE;
  if (batch == 0) return PQ_OK;
  if (!global_div || !scratch_tmax) return PQ_ERR_NULL;
  cudaStream_t stream = (cudaStream_t)stream_;
  int st = cuda_status(cudaMemsetAsync(scratch_tmax, 0, (size_t)batch * sizeof(uint32_t), stream));
  if (st) return st;
  st = pq_nvfp4_codes(w, batch, rows, cols, codes, scratch_amax, scratch_tmax, stream_);
  if (st) return st;
  const int64_t ng = rows * cols / 16;
  for (int64_t b0 = 0; b0 < batch; b0 += pq::MAX_SCALE_SLICES) {
    const int nb = (int)((batch - b0) < pq::MAX_SCALE_SLICES ? (batch - b0) : pq::MAX_SCALE_SLICES);
    std::vector<const uint16_t*> am(nb);
    std::vector<int64_t> ngs(nb, ng);
    std::vector<uint8_t*> sc(nb);
    for (int i = 0; i < nb; ++i) {
      am[i] = scratch_amax + (b0 + i) * ng;
      sc[i] = scales + (b0 + i) * ng;
    }
    st = pq_nvfp4_scales(nb, am.data(), ngs.data(), scratch_tmax + b0, nullptr,
                         override_dev ? override_dev + b0 : nullptr, sc.data(), global_div + b0, stream_);
    if (st) return st;
  }
  return PQ_OK;
}

int pq_nvfp4_global_real(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols, uint32_t* scratch,
                         float* global_real, void* stream) {
  if (batch < 0 || rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (cols % 16) return PQ_ERR_SHAPE;
  if (batch == 0) return PQ_OK;
  if (batch > pq::MAX_SCALE_SLICES) return PQ_ERR_LIMIT;
  if (!scratch || !global_real || (rows > 0 && !w)) return PQ_ERR_NULL;
  if (!aligned(w, 16) || !aligned(scratch, 4)) return PQ_ERR_ALIGN;
  return cuda_status(pq::launch_nvfp4_global(w, rows * cols, (int)batch, scratch, global_real, num_sms_current(),
                                             (cudaStream_t)stream));
}

int pq_mxfp8_pack(const uint16_t* w, int64_t n_rows, int64_t cols, uint8_t* q, uint8_t* scale_e8m0, void* stream) {
  if (n_rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (cols % 32) return PQ_ERR_SHAPE;
  if (n_rows == 0) return PQ_OK;
  if (!w || !q || !scale_e8m0) return PQ_ERR_NULL;
  if (!aligned(w, 16) || !aligned(q, 8)) return PQ_ERR_ALIGN;
  return cuda_status(pq::launch_mxfp8_pack(w, n_rows * cols, q, scale_e8m0, num_sms_current(), (cudaStream_t)stream));
}

int pq_fp8_channel_pack(const uint16_t* w, int64_t n_rows, int64_t cols, uint8_t* q, float* scale, void* stream) {
  if (n_rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (n_rows == 0) return PQ_OK;
  if (!w || !q || !scale) return PQ_ERR_NULL;
  if ((cols % 8) == 0 && (!aligned(w, 16) || !aligned(q, 8))) return PQ_ERR_ALIGN;
  return cuda_status(pq::launch_fp8_channel_pack(w, n_rows, cols, q, scale, num_sms_current(), (cudaStream_t)stream));
}

int pq_sumsq_rows(const uint16_t* g, int64_t n_rows, int64_t cols, double* total, float* per_row, void* stream) {
  if (n_rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (!total) return PQ_ERR_NULL;
  if (n_rows == 0) return PQ_OK;
  if (!g) return PQ_ERR_NULL;
  return cuda_status(pq::launch_sumsq_rows(g, n_rows, cols, total, per_row, num_sms_current(), (cudaStream_t)stream));
}

int pq_sumsq_rows_full(const uint16_t* g, int64_t n_rows, int64_t cols, double* total, float* per_row,
                       float* h_full, void* stream) {
  if (n_rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (!total || !h_full) return PQ_ERR_NULL;
  if (n_rows == 0) return PQ_OK;
  if (!g) return PQ_ERR_NULL;
  return cuda_status(
      pq::launch_sumsq_rows_full(g, n_rows, cols, total, per_row, h_full, num_sms_current(), (cudaStream_t)stream));
}

int pq_rownorm2(const uint16_t* x, int64_t T, int64_t d, float* out, void* stream) {
  if (T < 0 || d < 1) return PQ_ERR_SHAPE;
  if (T == 0) return PQ_OK;
  if (!x || !out) return PQ_ERR_NULL;
  return cuda_status(pq::launch_rownorm2(x, T, d, out, num_sms_current(), (cudaStream_t)stream));
}

int pq_tokennorm_dot(const uint16_t* g, int64_t T, int64_t d, const float* xnorm, const int64_t* token_idx,
                     double* acc, void* stream) {
  if (T < 0 || d < 1) return PQ_ERR_SHAPE;
  if (!acc) return PQ_ERR_NULL;
  if (T > 0 && (!g || !xnorm)) return PQ_ERR_NULL;
  return cuda_status(
      pq::launch_tokennorm_dot(g, T, d, xnorm, token_idx, acc, num_sms_current(), (cudaStream_t)stream));
}

int pq_tokennorm_dot_seg(const uint16_t* g, int64_t R, int64_t d, const float* xnorm, const int64_t* token_idx,
                         const int32_t* seg, int64_t n_seg, double* acc, void* stream) {
  if (R < 0 || d < 1 || n_seg < 0) return PQ_ERR_SHAPE;
  if (R == 0) return PQ_OK;
  if (!g || !xnorm || !seg || !acc) return PQ_ERR_NULL;
  return cuda_status(
      pq::launch_tokennorm_seg(g, R, d, xnorm, token_idx, seg, acc, num_sms_current(), (cudaStream_t)stream));
}

}  // extern "C"
