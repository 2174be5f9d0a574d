// C ABI of libbsp.so (declared in include/bsp.h).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "bsp_internal.h"

namespace bsp {

static thread_local std::string g_last_error;

bsp_status set_error(bsp_status s, const std::string& msg) {
  g_last_error = msg;
  return s;
}

bsp_status cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return BSP_OK;
  return set_error(BSP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bsp_status encode_2d(bsp_device* dev, CUtensorMap* tm, CUtensorMapDataType dt, int esize,
                     const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                     uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "device pointers must be 16-byte aligned");
  if ((row_stride_elems * esize) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "row strides must be multiples of 16 bytes");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_elems * static_cast<uint64_t>(esize)};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = dev->encode(tm, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(BSP_ERR_INVALID_ARG,
                     "cuTensorMapEncodeTiled failed (code " + std::to_string(int(r)) + ")");
  return BSP_OK;
}

bsp_status encode_nd(bsp_device* dev, CUtensorMap* tm, CUtensorMapDataType dt, int rank,
                     const void* ptr, const uint64_t* dims, const uint64_t* strides_bytes,
                     const uint32_t* box, CUtensorMapSwizzle swz) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "device pointers must be 16-byte aligned");
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i > 0) {
      if (strides_bytes[i - 1] % 16)
        return set_error(BSP_ERR_INVALID_ARG, "row strides must be multiples of 16 bytes");
      s[i - 1] = strides_bytes[i - 1];
    }
  }
  CUresult r = dev->encode(tm, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(ptr), d, s, b,
                           e, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(BSP_ERR_INVALID_ARG,
                     "cuTensorMapEncodeTiled (rank " + std::to_string(rank) + ") failed (code " +
                         std::to_string(int(r)) + ")");
  return BSP_OK;
}

static bsp_status check_desc(const bsp_bsr_desc* A, bool need_values) {
  if (!A) return set_error(BSP_ERR_INVALID_ARG, "null BSR descriptor");
  if (A->R <= 0 || A->C <= 0 || A->rows <= 0 || A->cols <= 0 || A->nnzb < 0)
    return set_error(BSP_ERR_INVALID_ARG, "bad BSR dimensions");
  if (A->rows % A->R || A->cols % A->C)
    return set_error(BSP_ERR_INVALID_ARG, "rows % R and cols % C must be 0");
  if (!A->row_ptr || (A->nnzb > 0 && !A->col_idx))
    return set_error(BSP_ERR_INVALID_ARG, "BSR row_ptr / col_idx missing");
  if (need_values && A->nnzb > 0 && !A->values)
    return set_error(BSP_ERR_INVALID_ARG, "BSR values missing");
  if (A->values && reinterpret_cast<uintptr_t>(A->values) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "BSR values must be 16-byte aligned");
  return BSP_OK;
}

// Pattern arrays on the host: use the caller's copies or fetch them.
static bsp_status host_pattern(const bsp_bsr_desc* A, const int32_t* hrp, const int32_t* hci,
                               std::vector<int32_t>* rp, std::vector<int32_t>* ci,
                               const int32_t** rp_out, const int32_t** ci_out) {
  const int64_t nbr = A->rows / A->R;
  if (hrp && (hci || A->nnzb == 0)) {
    *rp_out = hrp;
    *ci_out = hci;
    return BSP_OK;
  }
  rp->resize(nbr + 1);
  ci->resize(std::max<int64_t>(A->nnzb, 1));
  bsp_status s = cuda_check(cudaMemcpy(rp->data(), A->row_ptr, sizeof(int32_t) * (nbr + 1),
                                       cudaMemcpyDeviceToHost),
                            "copy row_ptr to host");
  if (s != BSP_OK) return s;
  if (A->nnzb > 0) {
    s = cuda_check(cudaMemcpy(ci->data(), A->col_idx, sizeof(int32_t) * A->nnzb,
                              cudaMemcpyDeviceToHost),
                   "copy col_idx to host");
    if (s != BSP_OK) return s;
  }
  *rp_out = rp->data();
  *ci_out = ci->data();
  return BSP_OK;
}

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Upload the plan tables as one device allocation.
static bsp_status upload_blob(const std::vector<std::pair<const void*, size_t>>& parts,
                              void** blob, size_t* bytes, std::vector<void*>* ptrs) {
  size_t total = 0;
  for (auto& pr : parts) total += align256(pr.second);
  total = std::max<size_t>(total, 256);
  void* d = nullptr;
  if (cudaMalloc(&d, total) != cudaSuccess)
    return set_error(BSP_ERR_ALLOC, "cudaMalloc of the plan tables failed");
  std::vector<uint8_t> h(total, 0);
  size_t off = 0;
  ptrs->clear();
  for (auto& pr : parts) {
    if (pr.second) memcpy(h.data() + off, pr.first, pr.second);
    ptrs->push_back(static_cast<uint8_t*>(d) + off);
    off += align256(pr.second);
  }
  cudaError_t e = cudaMemcpy(d, h.data(), total, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_check(e, "upload plan tables");
  }
  *blob = d;
  *bytes = total;
  return BSP_OK;
}

// Plan tables of a temporary plan of the host-buffer path: packed into the
// device's pinned staging and copied on `stream` into its plan area, both
// grow-only, so no per-call allocation, free or synchronous copy.  The caller
// synchronises before the next host-buffer call reuses them.
static bsp_status upload_blob_borrowed(bsp_device* dev,
                                       const std::vector<std::pair<const void*, size_t>>& parts,
                                       cudaStream_t stream, void** blob, size_t* bytes,
                                       std::vector<void*>* ptrs) {
  size_t total = 0;
  for (auto& pr : parts) total += align256(pr.second);
  total = std::max<size_t>(total, 256);
  if (dev->plan_ws_bytes < total) {
    if (dev->plan_ws) cudaFree(dev->plan_ws);
    dev->plan_ws = nullptr;
    dev->plan_ws_bytes = 0;
    if (cudaMalloc(&dev->plan_ws, total) != cudaSuccess)
      return set_error(BSP_ERR_ALLOC, "cudaMalloc of the plan-table area failed");
    dev->plan_ws_bytes = total;
  }
  if (dev->pinned_bytes < total) {
    if (dev->pinned) cudaFreeHost(dev->pinned);
    dev->pinned = nullptr;
    dev->pinned_bytes = 0;
    if (cudaHostAlloc(&dev->pinned, total, cudaHostAllocDefault) != cudaSuccess)
      return set_error(BSP_ERR_ALLOC, "cudaHostAlloc of the plan-table staging failed");
    dev->pinned_bytes = total;
  }
  uint8_t* h = static_cast<uint8_t*>(dev->pinned);
  size_t off = 0;
  ptrs->clear();
  for (auto& pr : parts) {
    if (pr.second) memcpy(h + off, pr.first, pr.second);
    ptrs->push_back(static_cast<uint8_t*>(dev->plan_ws) + off);
    off += align256(pr.second);
  }
  bsp_status st = cuda_check(cudaMemcpyAsync(dev->plan_ws, h, total, cudaMemcpyHostToDevice, stream),
                             "upload plan tables");
  if (st != BSP_OK) return st;
  *blob = dev->plan_ws;
  *bytes = total;
  return BSP_OK;
}

// Copy / compute streams and events of the host-buffer path (created once).
static bsp_status host_streams(bsp_device* dev, size_t n_events) {
  if (!dev->s_h2d) {
    bsp_status s = cuda_check(cudaStreamCreateWithFlags(&dev->s_h2d, cudaStreamNonBlocking), "cudaStreamCreate");
    if (s == BSP_OK) s = cuda_check(cudaStreamCreateWithFlags(&dev->s_comp, cudaStreamNonBlocking), "cudaStreamCreate");
    if (s == BSP_OK) s = cuda_check(cudaStreamCreateWithFlags(&dev->s_d2h, cudaStreamNonBlocking), "cudaStreamCreate");
    if (s != BSP_OK) return s;
  }
  while (dev->ev_in.size() < n_events) {
    cudaEvent_t a = nullptr, b = nullptr;
    bsp_status s = cuda_check(cudaEventCreateWithFlags(&a, cudaEventDisableTiming), "cudaEventCreate");
    if (s == BSP_OK) s = cuda_check(cudaEventCreateWithFlags(&b, cudaEventDisableTiming), "cudaEventCreate");
    if (s != BSP_OK) return s;
    dev->ev_in.push_back(a);
    dev->ev_out.push_back(b);
  }
  return BSP_OK;
}

static bsp_status ws_reserve(bsp_device* dev, size_t bytes) {
  if (dev->ws_bytes >= bytes) return BSP_OK;
  if (dev->ws) cudaFree(dev->ws);
  dev->ws = nullptr;
  dev->ws_bytes = 0;
  if (cudaMalloc(&dev->ws, bytes) != cudaSuccess)
    return set_error(BSP_ERR_ALLOC, "cudaMalloc of the host-path workspace failed");
  dev->ws_bytes = bytes;
  return BSP_OK;
}

}  // namespace bsp

using namespace bsp;

extern "C" {

const char* bsp_last_error_string(void) { return g_last_error.c_str(); }

const char* bsp_status_string(bsp_status s) {
  switch (s) {
    case BSP_OK: return "ok";
    case BSP_ERR_INVALID_ARG: return "invalid argument";
    case BSP_ERR_UNSUPPORTED: return "unsupported";
    case BSP_ERR_CUDA: return "cuda error";
    case BSP_ERR_TIMEOUT: return "device wait timed out";
    case BSP_ERR_NCCL: return "nccl error";
    case BSP_ERR_ALLOC: return "allocation failed";
    case BSP_ERR_STATE: return "bad state";
  }
  return "unknown";
}

bsp_status bsp_device_open(int ordinal, bsp_device** out) {
  if (!out) return set_error(BSP_ERR_INVALID_ARG, "null output");
  *out = nullptr;
  int n = 0;
  bsp_status s = cuda_check(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (s != BSP_OK) return s;
  if (ordinal < 0 || ordinal >= n) return set_error(BSP_ERR_INVALID_ARG, "no such device");
  s = cuda_check(cudaSetDevice(ordinal), "cudaSetDevice");
  if (s != BSP_OK) return s;
  cudaDeviceProp prop;
  s = cuda_check(cudaGetDeviceProperties(&prop, ordinal), "cudaGetDeviceProperties");
  if (s != BSP_OK) return s;
  if (prop.major != 10)
    return set_error(BSP_ERR_UNSUPPORTED, "libbsp is built for sm_100a (B200); this device is sm_" +
                                              std::to_string(prop.major * 10 + prop.minor));
  bsp_device* d = new (std::nothrow) bsp_device();
  if (!d) return set_error(BSP_ERR_ALLOC, "host allocation failed");
  d->ordinal = ordinal;
  d->sm_count = prop.multiProcessorCount;
  d->max_smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn) {
    delete d;
    return set_error(BSP_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
  }
  d->encode = reinterpret_cast<PFN_encodeTiled>(fn);
  if (cudaMalloc(&d->d_status, 64) != cudaSuccess) {
    delete d;
    return set_error(BSP_ERR_ALLOC, "cudaMalloc of the status word failed");
  }
  cudaMemset(d->d_status, 0, 64);
  *out = d;
  return BSP_OK;
}

bsp_status bsp_device_close(bsp_device* dev) {
  if (!dev) return BSP_OK;
  cudaSetDevice(dev->ordinal);
  if (dev->d_status) cudaFree(dev->d_status);
  if (dev->ws) cudaFree(dev->ws);
  if (dev->pinned) cudaFreeHost(dev->pinned);
  if (dev->plan_ws) cudaFree(dev->plan_ws);
  if (dev->aux_ws) cudaFree(dev->aux_ws);
  for (auto& sl : dev->batch_slots) {
    if (sl.d) cudaFree(sl.d);
    if (sl.h) cudaFreeHost(sl.h);
  }
  for (cudaEvent_t e : dev->ev_in) cudaEventDestroy(e);
  for (cudaEvent_t e : dev->ev_out) cudaEventDestroy(e);
  if (dev->s_h2d) cudaStreamDestroy(dev->s_h2d);
  if (dev->s_comp) cudaStreamDestroy(dev->s_comp);
  if (dev->s_d2h) cudaStreamDestroy(dev->s_d2h);
  delete dev;
  return BSP_OK;
}

int bsp_device_sm_count(const bsp_device* dev) { return dev ? dev->sm_count : 0; }

bsp_status bsp_device_get_error(bsp_device* dev, uint32_t* bits) {
  if (!dev || !bits) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  return cuda_check(cudaMemcpy(bits, dev->d_status, 4, cudaMemcpyDeviceToHost), "read status");
}

bsp_status bsp_device_synchronize(bsp_device* dev) {
  if (!dev) return set_error(BSP_ERR_INVALID_ARG, "null device");
  bsp_status s = cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  if (s != BSP_OK) return s;
  uint32_t bits = 0;
  s = cuda_check(cudaMemcpy(&bits, dev->d_status, 4, cudaMemcpyDeviceToHost), "read status");
  if (s != BSP_OK) return s;
  if (bits) {
    cudaMemset(dev->d_status, 0, 4);
    char msg[128];
    snprintf(msg, sizeof(msg), "a kernel wait timed out (status bits 0x%x)", bits);
    return set_error(BSP_ERR_TIMEOUT, msg);
  }
  return BSP_OK;
}

// ------------------------------------------------ device storage ----
namespace {
struct OnDevice {  // make `ordinal` current for a call, put the caller's device back after
  int prev = -1;
  explicit OnDevice(int ordinal) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != ordinal) cudaSetDevice(ordinal);
  }
  ~OnDevice() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace

bsp_status bsp_buffer_alloc(bsp_device* dev, int64_t bytes, void** ptr) {
  if (!dev || !ptr || bytes < 0) return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  *ptr = nullptr;
  OnDevice on(dev->ordinal);
  if (cudaMalloc(ptr, static_cast<size_t>(std::max<int64_t>(bytes, 1))) != cudaSuccess) {
    *ptr = nullptr;
    return set_error(BSP_ERR_ALLOC, "cudaMalloc of " + std::to_string(bytes) + " bytes failed");
  }
  return BSP_OK;
}

bsp_status bsp_buffer_free(bsp_device* dev, void* ptr) {
  if (!dev) return set_error(BSP_ERR_INVALID_ARG, "null device");
  if (!ptr) return BSP_OK;
  OnDevice on(dev->ordinal);
  return cuda_check(cudaFree(ptr), "cudaFree");
}

bsp_status bsp_buffer_write(bsp_device* dev, void* dst, const void* src, int64_t bytes) {
  if (!dev || (bytes > 0 && (!dst || !src)) || bytes < 0) return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  if (bytes == 0) return BSP_OK;
  OnDevice on(dev->ordinal);
  return cuda_check(cudaMemcpy(dst, src, static_cast<size_t>(bytes), cudaMemcpyHostToDevice), "buffer write");
}

bsp_status bsp_buffer_read(bsp_device* dev, void* dst, const void* src, int64_t bytes) {
  if (!dev || (bytes > 0 && (!dst || !src)) || bytes < 0) return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  if (bytes == 0) return BSP_OK;
  OnDevice on(dev->ordinal);
  return cuda_check(cudaMemcpy(dst, src, static_cast<size_t>(bytes), cudaMemcpyDeviceToHost), "buffer read");
}

bsp_status bsp_bsr_upload(bsp_device* dev, int64_t rows, int64_t cols, int32_t R, int32_t C, int64_t nnzb,
                          const int32_t* host_row_ptr, const int32_t* host_col_idx, const uint16_t* host_values,
                          bsp_bsr_desc* out) {
  if (!dev || !out || !host_row_ptr || (nnzb > 0 && !host_col_idx))
    return set_error(BSP_ERR_INVALID_ARG, "null argument");
  memset(out, 0, sizeof(*out));
  if (R <= 0 || C <= 0 || rows <= 0 || cols <= 0 || nnzb < 0 || rows % R || cols % C)
    return set_error(BSP_ERR_INVALID_ARG, "bad BSR shape (rows % R and cols % C must be 0)");
  const int64_t nbr = rows / R, nbc = cols / C;
  if (host_row_ptr[0] != 0 || host_row_ptr[nbr] != nnzb)
    return set_error(BSP_ERR_INVALID_ARG, "row_ptr must start at 0 and end at nnzb");
  for (int64_t i = 0; i < nbr; ++i)
    if (host_row_ptr[i + 1] < host_row_ptr[i]) return set_error(BSP_ERR_INVALID_ARG, "row_ptr must not decrease");
  for (int64_t b = 0; b < nnzb; ++b)
    if (host_col_idx[b] < 0 || host_col_idx[b] >= nbc)
      return set_error(BSP_ERR_INVALID_ARG, "column index out of range");
  // one allocation: row_ptr at its start, col_idx, then the values at a
  // 256-byte boundary (TMA wants 16, the kernels' boxes read 128-byte rows)
  const size_t rp_bytes = sizeof(int32_t) * static_cast<size_t>(nbr + 1);
  const size_t ci_off = align256(rp_bytes);
  const size_t ci_bytes = sizeof(int32_t) * static_cast<size_t>(std::max<int64_t>(nnzb, 1));
  const size_t v_off = ci_off + align256(ci_bytes);
  const size_t v_bytes = host_values ? 2 * static_cast<size_t>(nnzb) * R * C : 0;
  OnDevice on(dev->ordinal);
  void* base = nullptr;
  if (cudaMalloc(&base, v_off + std::max<size_t>(v_bytes, 16)) != cudaSuccess)
    return set_error(BSP_ERR_ALLOC, "cudaMalloc of the BSR matrix failed");
  uint8_t* b8 = static_cast<uint8_t*>(base);
  bsp_status s = cuda_check(cudaMemcpy(b8, host_row_ptr, rp_bytes, cudaMemcpyHostToDevice), "upload row_ptr");
  if (s == BSP_OK && nnzb > 0)
    s = cuda_check(cudaMemcpy(b8 + ci_off, host_col_idx, sizeof(int32_t) * nnzb, cudaMemcpyHostToDevice),
                   "upload col_idx");
  if (s == BSP_OK && v_bytes > 0)
    s = cuda_check(cudaMemcpy(b8 + v_off, host_values, v_bytes, cudaMemcpyHostToDevice), "upload values");
  if (s != BSP_OK) {
    cudaFree(base);
    return s;
  }
  out->rows = rows;
  out->cols = cols;
  out->R = R;
  out->C = C;
  out->nnzb = nnzb;
  out->row_ptr = reinterpret_cast<const int32_t*>(b8);
  out->col_idx = reinterpret_cast<const int32_t*>(b8 + ci_off);
  out->values = host_values ? b8 + v_off : nullptr;
  return BSP_OK;
}

bsp_status bsp_bsr_free(bsp_device* dev, bsp_bsr_desc* desc) {
  if (!dev || !desc) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  bsp_status s = BSP_OK;
  if (desc->row_ptr) {
    OnDevice on(dev->ordinal);
    s = cuda_check(cudaFree(const_cast<int32_t*>(desc->row_ptr)), "cudaFree (BSR)");
  }
  memset(desc, 0, sizeof(*desc));
  return s;
}

// ---------------------------------------------------------------- SpMM ----
// Plan creation; `borrow` (host-buffer path only) keeps the tables in the
// device's plan area, uploaded on `stream`.
static bsp_status spmm_plan_create_impl(bsp_device* dev, const bsp_bsr_desc* A, const int32_t* host_row_ptr,
                                        const int32_t* host_col_idx, int64_t N, bsp_dtype c_type,
                                        bsp_strategy strategy, const bsp_spmm_opts* opts, bool borrow,
                                        cudaStream_t stream, bsp_spmm_plan** out);

bsp_status bsp_spmm_plan_create(bsp_device* dev, const bsp_bsr_desc* A, const int32_t* host_row_ptr,
                                const int32_t* host_col_idx, int64_t N, bsp_dtype c_type,
                                bsp_strategy strategy, const bsp_spmm_opts* opts,
                                bsp_spmm_plan** out) {
  return spmm_plan_create_impl(dev, A, host_row_ptr, host_col_idx, N, c_type, strategy, opts, false, nullptr,
                               out);
}

// The device tables of a planned SpMM, in upload order: units, CTA offsets,
// steps, stage list, CTA stage offsets, and two zeroed sets of split-K
// counters (used by alternate launches; each launch zeroes the other set).
static std::vector<std::pair<const void*, size_t>> spmm_table_parts(const bsp_spmm_plan& p,
                                                                    std::vector<int32_t>* zeros) {
  zeros->assign(2 * static_cast<size_t>(p.n_split_slots), 0);
  return {{p.h_units.data(), p.h_units.size() * sizeof(SpmmUnit)},
          {p.h_cta_begin.data(), p.h_cta_begin.size() * sizeof(int32_t)},
          {p.h_steps.data(), p.h_steps.size() * sizeof(int32_t)},
          {p.h_stage_list.data(), p.h_stage_list.size() * sizeof(int32_t)},
          {p.h_cta_stage_begin.data(), p.h_cta_stage_begin.size() * sizeof(int32_t)},
          {zeros->data(), zeros->size() * sizeof(int32_t)},
          {p.h_entry_rows.data(), p.h_entry_rows.size() * sizeof(int32_t)}};
}

static void spmm_bind_tables(bsp_spmm_plan* p, const std::vector<void*>& ptrs) {
  p->d_units = static_cast<SpmmUnit*>(ptrs[0]);
  p->d_cta_begin = static_cast<int32_t*>(ptrs[1]);
  p->d_steps = static_cast<int32_t*>(ptrs[2]);
  p->d_stage_list = static_cast<int4*>(ptrs[3]);
  p->d_cta_stage_begin = static_cast<int32_t*>(ptrs[4]);
  p->d_split_counters = static_cast<int32_t*>(ptrs[5]);
  p->d_entry_rows = p->h_entry_rows.empty() ? nullptr : static_cast<int32_t*>(ptrs[6]);
}

// Bytes of the split-K partial tiles: 128 rows x the tile's accumulator
// columns, fp32, per workspace slot.
static size_t spmm_split_ws_bytes(const bsp_spmm_plan& p) {
  const int64_t acc_cols = p.variant >= 2 ? 256 : 128 * p.NT;
  return sizeof(float) * 128 * static_cast<size_t>(acc_cols) * static_cast<size_t>(p.n_split_slots);
}

static bsp_status spmm_plan_create_impl(bsp_device* dev, const bsp_bsr_desc* A, const int32_t* host_row_ptr,
                                        const int32_t* host_col_idx, int64_t N, bsp_dtype c_type,
                                        bsp_strategy strategy, const bsp_spmm_opts* opts, bool borrow,
                                        cudaStream_t stream, bsp_spmm_plan** out) {
  if (!dev || !out) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  bsp_status s = check_desc(A, false);
  if (s != BSP_OK) return s;
  if (c_type != BSP_BF16 && c_type != BSP_F32)
    return set_error(BSP_ERR_INVALID_ARG, "C type must be BSP_BF16 or BSP_F32");
  std::vector<int32_t> rp, ci;
  const int32_t *prp = nullptr, *pci = nullptr;
  s = host_pattern(A, host_row_ptr, host_col_idx, &rp, &ci, &prp, &pci);
  if (s != BSP_OK) return s;
  bsp_spmm_plan* p = new (std::nothrow) bsp_spmm_plan();
  if (!p) return set_error(BSP_ERR_ALLOC, "host allocation failed");
  p->dev = dev;
  p->M = A->rows;
  p->K = A->cols;
  p->N = N;
  p->R = A->R;
  p->C = A->C;
  p->nnzb = A->nnzb;
  p->c_type = c_type;
  p->strategy = strategy;
  s = plan_spmm_host(p, prp, pci, dev->sm_count, dev->max_smem_optin, opts);
  if (s != BSP_OK) {
    delete p;
    return s;
  }
  std::vector<void*> ptrs;
  std::vector<int32_t> zeros;
  const auto parts = spmm_table_parts(*p, &zeros);
  s = borrow ? upload_blob_borrowed(dev, parts, stream, &p->d_blob, &p->blob_bytes, &ptrs)
             : upload_blob(parts, &p->d_blob, &p->blob_bytes, &ptrs);
  p->blob_borrowed = borrow;
  if (s != BSP_OK) {
    delete p;
    return s;
  }
  spmm_bind_tables(p, ptrs);
  if (p->n_split_slots > 0) {
    const size_t wb = spmm_split_ws_bytes(*p);
    if (borrow) {
      if (dev->aux_ws_bytes < wb) {
        if (dev->aux_ws) cudaFree(dev->aux_ws);
        dev->aux_ws = nullptr;
        dev->aux_ws_bytes = 0;
        if (cudaMalloc(&dev->aux_ws, wb) != cudaSuccess) {
          bsp_spmm_plan_destroy(p);
          return set_error(BSP_ERR_ALLOC, "cudaMalloc of the split-K workspace failed");
        }
        dev->aux_ws_bytes = wb;
      }
      p->d_split_ws = static_cast<float*>(dev->aux_ws);
    } else if (cudaMalloc(reinterpret_cast<void**>(&p->d_split_ws), wb) != cudaSuccess) {
      bsp_spmm_plan_destroy(p);
      return set_error(BSP_ERR_ALLOC, "cudaMalloc of the split-K workspace failed");
    }
  }
  *out = p;
  return BSP_OK;
}

bsp_status bsp_spmm_execute(const bsp_spmm_plan* plan, const bsp_bsr_desc* A, const void* B,
                            int64_t ldb, void* C, int64_t ldc, void* stream) {
  if (!plan || !B || !C) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  bsp_status s = check_desc(A, true);
  if (s != BSP_OK) return s;
  if (A->rows != plan->M || A->cols != plan->K || A->R != plan->R || A->C != plan->C ||
      A->nnzb != plan->nnzb)
    return set_error(BSP_ERR_INVALID_ARG, "A does not match the plan's pattern");
  if (ldb < plan->N || ldc < plan->N)
    return set_error(BSP_ERR_INVALID_ARG, "leading dimensions must be >= N");
  if (plan->variant == 2 || plan->variant == 3)
    return launch_spmm_pair(plan, A, B, ldb, C, ldc, static_cast<cudaStream_t>(stream));
  if (plan->variant == 1)
    return launch_spmm_rowstack(plan, A, B, ldb, C, ldc, static_cast<cudaStream_t>(stream));
  return launch_spmm(plan, A, B, ldb, C, ldc, static_cast<cudaStream_t>(stream));
}

bsp_status bsp_spmm_execute_replicated(const bsp_spmm_plan* plan, const bsp_bsr_desc* A, const void* B,
                                       int64_t ldb, void* C, int64_t ldc, void* const* peer_C,
                                       int32_t n_peers, void* stream) {
  if (!plan || !B || !C) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  bsp_status s = check_desc(A, true);
  if (s != BSP_OK) return s;
  if (A->rows != plan->M || A->cols != plan->K || A->R != plan->R || A->C != plan->C ||
      A->nnzb != plan->nnzb)
    return set_error(BSP_ERR_INVALID_ARG, "A does not match the plan's pattern");
  if (ldb < plan->N || ldc < plan->N)
    return set_error(BSP_ERR_INVALID_ARG, "leading dimensions must be >= N");
  if (plan->variant == 2 || plan->variant == 3)
    return launch_spmm_pair(plan, A, B, ldb, C, ldc, static_cast<cudaStream_t>(stream), peer_C, n_peers);
  if (plan->variant != 1)
    return set_error(BSP_ERR_UNSUPPORTED, "replicated output needs a DDA (row-stacked) plan");
  return launch_spmm_rowstack(plan, A, B, ldb, C, ldc, static_cast<cudaStream_t>(stream), peer_C,
                              n_peers);
}

// ---- CUDA IPC of output buffers (replicated multi-GPU output) --------------
namespace {
typedef CUresult (*PFN_getAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

struct DeviceScope {  // make dev current for the call, restore the caller's device after
  int prev = -1;
  explicit DeviceScope(int ordinal) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != ordinal) cudaSetDevice(ordinal);
  }
  ~DeviceScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace

bsp_status bsp_ipc_export(bsp_device* dev, const void* ptr, void* handle_out, int64_t* offset_out) {
  if (!dev || !ptr || !handle_out || !offset_out) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  DeviceScope scope(dev->ordinal);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn)
    return set_error(BSP_ERR_CUDA, "cuMemGetAddressRange not available from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (reinterpret_cast<PFN_getAddressRange>(fn)(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(BSP_ERR_INVALID_ARG, "pointer is not device memory of this process");
  cudaIpcMemHandle_t h;
  bsp_status s = cuda_check(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  if (s != BSP_OK) return s;
  static_assert(sizeof(h) == BSP_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return BSP_OK;
}

bsp_status bsp_ipc_import(bsp_device* dev, const void* handle, void** base_out) {
  if (!dev || !handle || !base_out) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  DeviceScope scope(dev->ordinal);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_check(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess),
                    "cudaIpcOpenMemHandle");
}

bsp_status bsp_ipc_close(bsp_device* dev, void* base) {
  if (!dev || !base) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  DeviceScope scope(dev->ordinal);
  return cuda_check(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}

bsp_status bsp_spmm_plan_destroy(bsp_spmm_plan* plan) {
  if (!plan) return BSP_OK;
  if (plan->d_blob && !plan->blob_borrowed) cudaFree(plan->d_blob);
  if (plan->d_split_ws && !plan->blob_borrowed) cudaFree(plan->d_split_ws);
  delete plan;
  return BSP_OK;
}

bsp_status bsp_spmm_plan_info(const bsp_spmm_plan* p, int64_t info[16]) {
  if (!p || !info) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  memset(info, 0, sizeof(int64_t) * 16);
  info[0] = p->n_units;
  info[1] = p->grid;
  info[2] = p->G;
  info[3] = p->NT;
  info[4] = p->Rs;
  info[5] = p->kc;
  info[6] = p->stages;
  info[7] = p->n_steps;
  info[8] = static_cast<int64_t>(p->blob_bytes);
  info[9] = p->smem_bytes;
  info[10] = p->tmem_cols;
  info[11] = p->variant;
  info[12] = p->nprod;
  info[15] = p->step_stride;  // int32 words per step-table entry
  return BSP_OK;
}

bsp_status bsp_spmm(bsp_device* dev, const bsp_bsr_desc* A, const void* B, int64_t ldb, void* C,
                    int64_t ldc, bsp_dtype c_type, int64_t N, bsp_strategy strategy,
                    const bsp_spmm_opts* opts, void* stream) {
  bsp_spmm_plan* p = nullptr;
  bsp_status s = bsp_spmm_plan_create(dev, A, nullptr, nullptr, N, c_type, strategy, opts, &p);
  if (s != BSP_OK) return s;
  s = bsp_spmm_execute(p, A, B, ldb, C, ldc, stream);
  if (s == BSP_OK) s = cuda_check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "sync");
  bsp_spmm_plan_destroy(p);
  if (s == BSP_OK) s = bsp_device_synchronize(dev);
  return s;
}

// Run `iters` timed launches after the first one; mean device ms per launch.
static bsp_status time_launches(int32_t iters, double* ms_out, cudaStream_t stream,
                                bsp_status (*launch)(const void*), const void* ctx) {
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  bsp_status s = cuda_check(cudaEventCreate(&e0), "cudaEventCreate");
  if (s == BSP_OK) s = cuda_check(cudaEventCreate(&e1), "cudaEventCreate");
  if (s == BSP_OK) s = cuda_check(cudaEventRecord(e0, stream), "cudaEventRecord");
  for (int32_t i = 0; s == BSP_OK && i < iters; ++i) s = launch(ctx);
  if (s == BSP_OK) s = cuda_check(cudaEventRecord(e1, stream), "cudaEventRecord");
  if (s == BSP_OK) s = cuda_check(cudaEventSynchronize(e1), "cudaEventSynchronize");
  float ms = 0.f;
  if (s == BSP_OK) s = cuda_check(cudaEventElapsedTime(&ms, e0, e1), "cudaEventElapsedTime");
  if (s == BSP_OK && ms_out) *ms_out = iters > 0 ? ms / iters : 0.0;
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  return s;
}

struct SpmmLaunchCtx {
  const bsp_spmm_plan* p;
  const bsp_bsr_desc* A;
  const void* B;
  void* C;
  int64_t N;
  cudaStream_t stream;
};
static bsp_status spmm_launch_ctx(const void* v) {
  const SpmmLaunchCtx* c = static_cast<const SpmmLaunchCtx*>(v);
  return bsp_spmm_execute(c->p, c->A, c->B, c->N, c->C, c->N, c->stream);
}

static bsp_status spmm_host_impl(bsp_device* dev, int64_t M, int64_t K, int32_t R, int32_t C,
                                 int64_t nnzb, const int32_t* row_ptr, const int32_t* col_idx,
                                 const uint16_t* values, const uint16_t* B, int64_t N,
                                 uint16_t* C_out, bsp_strategy strategy, const bsp_spmm_opts* opts,
                                 int32_t iters, double* ms_out) {
  if (!dev || !row_ptr || !B || !C_out || (nnzb > 0 && (!col_idx || !values)))
    return set_error(BSP_ERR_INVALID_ARG, "null argument");
  if (R <= 0 || C <= 0 || M % R || K % C) return set_error(BSP_ERR_INVALID_ARG, "bad dimensions");
  const int64_t nbr = M / R;
  const size_t b_val = align256(sizeof(uint16_t) * nnzb * R * C);
  const size_t b_rp = align256(sizeof(int32_t) * (nbr + 1));
  const size_t b_ci = align256(sizeof(int32_t) * std::max<int64_t>(nnzb, 1));
  const size_t b_B = align256(sizeof(uint16_t) * K * N);
  const size_t b_C = align256(sizeof(uint16_t) * M * N);
  bsp_status s = ws_reserve(dev, b_val + b_rp + b_ci + b_B + b_C);
  if (s != BSP_OK) return s;
  // Column panels of B and C: the copy of panel j + 1 in and of panel j - 1
  // out overlap panel j's kernel (the copy engines run both directions at
  // once).  Profiling calls time one whole-width kernel instead.
  int P = 1;
  if (iters == 0)
    for (int q : {4, 2})
      if (N % (256 * q) == 0 && N / q >= 512) {
        P = q;
        break;
      }
  const int64_t Np = N / P;
  s = host_streams(dev, static_cast<size_t>(P));
  if (s != BSP_OK) return s;
  uint8_t* w = static_cast<uint8_t*>(dev->ws);
  void* d_val = w;
  int32_t* d_rp = reinterpret_cast<int32_t*>(w + b_val);
  int32_t* d_ci = reinterpret_cast<int32_t*>(w + b_val + b_rp);
  uint16_t* d_B = reinterpret_cast<uint16_t*>(w + b_val + b_rp + b_ci);
  uint16_t* d_C = reinterpret_cast<uint16_t*>(w + b_val + b_rp + b_ci + b_B);
  cudaStream_t sh = dev->s_h2d, sc = dev->s_comp, sd = dev->s_d2h;
  const size_t pitch = sizeof(uint16_t) * N, pw = sizeof(uint16_t) * Np;
  auto run = [&]() -> bsp_status {
    bsp_status st;
    if ((st = cuda_check(cudaMemcpyAsync(d_rp, row_ptr, sizeof(int32_t) * (nbr + 1), cudaMemcpyHostToDevice, sh), "H2D row_ptr")) != BSP_OK) return st;
    if (nnzb > 0) {
      if ((st = cuda_check(cudaMemcpyAsync(d_ci, col_idx, sizeof(int32_t) * nnzb, cudaMemcpyHostToDevice, sh), "H2D col_idx")) != BSP_OK) return st;
      if ((st = cuda_check(cudaMemcpyAsync(d_val, values, sizeof(uint16_t) * nnzb * R * C, cudaMemcpyHostToDevice, sh), "H2D values")) != BSP_OK) return st;
    }
    for (int j = 0; j < P; ++j) {
      if ((st = cuda_check(cudaMemcpy2DAsync(d_B + j * Np, pitch, B + j * Np, pitch, pw, K, cudaMemcpyHostToDevice, sh), "H2D B")) != BSP_OK) return st;
      if ((st = cuda_check(cudaEventRecord(dev->ev_in[j], sh), "cudaEventRecord")) != BSP_OK) return st;
    }
    // the plan is built on the host while B streams in
    bsp_bsr_desc A{M, K, R, C, nnzb, d_rp, d_ci, d_val};
    bsp_spmm_plan* p = nullptr;
    st = spmm_plan_create_impl(dev, &A, row_ptr, col_idx, Np, BSP_BF16, strategy, opts, true, sc, &p);
    if (st != BSP_OK) return st;
    for (int j = 0; j < P && st == BSP_OK; ++j) {
      st = cuda_check(cudaStreamWaitEvent(sc, dev->ev_in[j], 0), "cudaStreamWaitEvent");
      if (st == BSP_OK) st = bsp_spmm_execute(p, &A, d_B + j * Np, N, d_C + j * Np, N, sc);
      if (st == BSP_OK) st = cuda_check(cudaEventRecord(dev->ev_out[j], sc), "cudaEventRecord");
      if (st == BSP_OK) st = cuda_check(cudaStreamWaitEvent(sd, dev->ev_out[j], 0), "cudaStreamWaitEvent");
      if (st == BSP_OK)
        st = cuda_check(cudaMemcpy2DAsync(C_out + j * Np, pitch, d_C + j * Np, pitch, pw, M, cudaMemcpyDeviceToHost, sd), "D2H C");
    }
    if (st == BSP_OK && iters > 0) {
      const SpmmLaunchCtx ctx{p, &A, d_B, d_C, N, sc};
      st = time_launches(iters, ms_out, sc, spmm_launch_ctx, &ctx);
    }
    if (st == BSP_OK) st = cuda_check(cudaStreamSynchronize(sd), "sync");
    if (st == BSP_OK) st = cuda_check(cudaStreamSynchronize(sc), "sync");
    bsp_spmm_plan_destroy(p);
    return st;
  };
  s = run();
  if (s != BSP_OK) {
    // nothing of this call may still run when the workspace is reused
    cudaStreamSynchronize(sh);
    cudaStreamSynchronize(sc);
    cudaStreamSynchronize(sd);
    return s;
  }
  return bsp_device_synchronize(dev);
}

bsp_status bsp_spmm_host(bsp_device* dev, int64_t M, int64_t K, int32_t R, int32_t C, int64_t nnzb,
                         const int32_t* row_ptr, const int32_t* col_idx, const uint16_t* values,
                         const uint16_t* B, int64_t N, uint16_t* C_out, bsp_strategy strategy,
                         const bsp_spmm_opts* opts) {
  return spmm_host_impl(dev, M, K, R, C, nnzb, row_ptr, col_idx, values, B, N, C_out, strategy,
                        opts, 0, nullptr);
}

// Copies n16 16-byte words from mapped pinned host memory into device memory
// with the SMs rather than a copy engine, so that a small plan table does not
// queue behind the large input copies already on the engine.
__global__ void fetch_mapped_words(uint4* __restrict__ dst, const uint4* __restrict__ src, size_t n16) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

bsp_status bsp_spmm_host_batch(bsp_device* dev, int32_t n_jobs, const bsp_spmm_host_job* jobs,
                               bsp_strategy strategy, const bsp_spmm_opts* opts) {
  if (!dev || n_jobs < 0 || (n_jobs > 0 && !jobs)) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  if (n_jobs == 0) return BSP_OK;
  const size_t nj = static_cast<size_t>(n_jobs);
  // device layout of each job: values | row_ptr | col_idx | B | C
  std::vector<size_t> off(nj + 1, 0);
  for (size_t k = 0; k < nj; ++k) {
    const bsp_spmm_host_job& j = jobs[k];
    if (!j.row_ptr || !j.B || !j.C_out || (j.nnzb > 0 && (!j.col_idx || !j.values)))
      return set_error(BSP_ERR_INVALID_ARG, "job " + std::to_string(k) + ": null argument");
    if (j.R <= 0 || j.C <= 0 || j.M <= 0 || j.K <= 0 || j.N <= 0 || j.M % j.R || j.K % j.C || j.nnzb < 0)
      return set_error(BSP_ERR_INVALID_ARG, "job " + std::to_string(k) + ": bad dimensions");
    off[k + 1] = off[k] + align256(sizeof(uint16_t) * j.nnzb * j.R * j.C) +
                 align256(sizeof(int32_t) * (j.M / j.R + 1)) + align256(sizeof(int32_t) * std::max<int64_t>(j.nnzb, 1)) +
                 align256(sizeof(uint16_t) * j.K * j.N) + align256(sizeof(uint16_t) * j.M * j.N);
  }
  bsp_status s = ws_reserve(dev, off[nj]);
  if (s == BSP_OK) s = host_streams(dev, 4 * nj);
  if (s != BSP_OK) return s;
  if (dev->batch_slots.size() < nj) dev->batch_slots.resize(nj);
  // A wide job runs as 2 or 4 column panels of one plan (whole 256-column
  // tiles; 2 panels from N = 1024, 4 from N = 8192): the first panel's
  // kernel starts when that panel of B is in, and each panel of C goes back
  // while later panels of B still arrive, so less of the step is spent with
  // one copy direction idle (the sweep's e2e: 24 -> 25 TF/s; four panels of
  // its N = 4096 measured no better than two).
  std::vector<int> panels(nj, 1);
  for (size_t k = 0; k < nj; ++k) {
    const int64_t n = jobs[k].N;
    if (n % 2048 == 0 && n >= 8192) panels[k] = 4;
    else if (n % 512 == 0 && n >= 1024) panels[k] = 2;
  }
  cudaStream_t sh = dev->s_h2d, sc = dev->s_comp, sd = dev->s_d2h;
  struct Dev {
    void* val;
    int32_t *rp, *ci;
    uint16_t *B, *C;
  };
  std::vector<Dev> d(nj);
  std::vector<bsp_spmm_plan*> plans(nj, nullptr);
  for (size_t k = 0; k < nj; ++k) {
    const bsp_spmm_host_job& j = jobs[k];
    bsp_spmm_plan* p = new (std::nothrow) bsp_spmm_plan();
    if (!p) {
      for (bsp_spmm_plan* q : plans) delete q;
      return set_error(BSP_ERR_ALLOC, "host allocation failed");
    }
    plans[k] = p;
    p->dev = dev;
    p->M = j.M;
    p->K = j.K;
    p->N = j.N / panels[k];
    p->R = j.R;
    p->C = j.C;
    p->nnzb = j.nnzb;
    p->c_type = BSP_BF16;
    p->strategy = strategy;
  }
  // 1. every job is planned on its own host thread from the start
  std::vector<bsp_status> pst(nj, BSP_OK);
  std::vector<std::string> pmsg(nj);
  std::vector<std::thread> th;
  // the jobs' planners share the cores
  static const int cores = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  const int cap = std::max(1, cores / static_cast<int>(nj));
  for (size_t k = 0; k < nj; ++k)
    th.emplace_back([&, k, cap]() {
      set_planner_thread_cap(cap);
      pst[k] = plan_spmm_host(plans[k], jobs[k].row_ptr, jobs[k].col_idx, dev->sm_count, dev->max_smem_optin, opts);
      if (pst[k] != BSP_OK) pmsg[k] = g_last_error;  // this worker's message
    });
  size_t joined = 0;
  auto join_upto = [&](size_t k) {  // threads 0..k done
    for (; joined <= k && joined < nj; ++joined) th[joined].join();
  };
  size_t queued = 0;  // jobs whose inputs are queued on the copy stream
  auto queue_inputs = [&](size_t k) -> bsp_status {
    const bsp_spmm_host_job& j = jobs[k];
    uint8_t* w = static_cast<uint8_t*>(dev->ws) + off[k];
    const size_t b_val = align256(sizeof(uint16_t) * j.nnzb * j.R * j.C);
    const size_t b_rp = align256(sizeof(int32_t) * (j.M / j.R + 1));
    const size_t b_ci = align256(sizeof(int32_t) * std::max<int64_t>(j.nnzb, 1));
    const size_t b_B = align256(sizeof(uint16_t) * j.K * j.N);
    d[k] = Dev{w, reinterpret_cast<int32_t*>(w + b_val), reinterpret_cast<int32_t*>(w + b_val + b_rp),
               reinterpret_cast<uint16_t*>(w + b_val + b_rp + b_ci),
               reinterpret_cast<uint16_t*>(w + b_val + b_rp + b_ci + b_B)};
    bsp_status st = cuda_check(cudaMemcpyAsync(d[k].rp, j.row_ptr, sizeof(int32_t) * (j.M / j.R + 1),
                                               cudaMemcpyHostToDevice, sh), "H2D row_ptr");
    if (st == BSP_OK && j.nnzb > 0)
      st = cuda_check(cudaMemcpyAsync(d[k].ci, j.col_idx, sizeof(int32_t) * j.nnzb, cudaMemcpyHostToDevice, sh),
                      "H2D col_idx");
    if (st == BSP_OK && j.nnzb > 0)
      st = cuda_check(cudaMemcpyAsync(d[k].val, j.values, sizeof(uint16_t) * j.nnzb * j.R * j.C,
                                      cudaMemcpyHostToDevice, sh), "H2D values");
    if (panels[k] == 1) {
      if (st == BSP_OK)
        st = cuda_check(cudaMemcpyAsync(d[k].B, j.B, sizeof(uint16_t) * j.K * j.N, cudaMemcpyHostToDevice, sh),
                        "H2D B");
      if (st == BSP_OK) st = cuda_check(cudaEventRecord(dev->ev_in[4 * k], sh), "cudaEventRecord");
    } else {
      const size_t pitch = sizeof(uint16_t) * static_cast<size_t>(j.N), part = pitch / panels[k];
      for (int h = 0; h < panels[k] && st == BSP_OK; ++h) {
        st = cuda_check(cudaMemcpy2DAsync(reinterpret_cast<uint8_t*>(d[k].B) + h * part, pitch,
                                          reinterpret_cast<const uint8_t*>(j.B) + h * part, pitch, part,
                                          static_cast<size_t>(j.K), cudaMemcpyHostToDevice, sh),
                        "H2D B panel");
        if (st == BSP_OK) st = cuda_check(cudaEventRecord(dev->ev_in[4 * k + h], sh), "cudaEventRecord");
      }
    }
    return st;
  };
  auto run = [&]() -> bsp_status {
    bsp_status st = BSP_OK;
    // 2. every job's inputs go onto the copy stream at once
    for (; queued < nj && st == BSP_OK; ++queued) st = queue_inputs(queued);
    for (size_t k = 0; k < nj && st == BSP_OK; ++k) {
      join_upto(k);
      bsp_spmm_plan* p = plans[k];
      p->blob_borrowed = true;  // after planning: the planner may replace the plan object (CTA pairs)
      if (pst[k] != BSP_OK) return set_error(pst[k], "job " + std::to_string(k) + ": " + pmsg[k]);
      // 3. job k's tables (and split-K partials) in its slot; the tables are
      //    fetched from mapped pinned memory by a small kernel on the compute
      //    stream, not queued behind the input copies on the copy engine
      std::vector<int32_t> zeros;
      const auto parts = spmm_table_parts(*p, &zeros);
      size_t tb = 0;
      for (auto& pr : parts) tb += align256(pr.second);
      tb = std::max<size_t>(tb, 256);
      const size_t sw = p->n_split_slots > 0 ? spmm_split_ws_bytes(*p) : 0;
      bsp_device::BatchSlot& sl = dev->batch_slots[k];
      if (sl.d_bytes < tb + sw) {
        if (sl.d) cudaFree(sl.d);  // synchronises: only while the slot grows
        sl.d = nullptr;
        sl.d_bytes = 0;
        if (cudaMalloc(&sl.d, tb + sw) != cudaSuccess) return set_error(BSP_ERR_ALLOC, "cudaMalloc of a batch slot failed");
        sl.d_bytes = tb + sw;
      }
      if (sl.h_bytes < tb) {
        if (sl.h) cudaFreeHost(sl.h);
        sl.h = nullptr;
        sl.h_bytes = 0;
        if (cudaHostAlloc(&sl.h, tb, cudaHostAllocMapped) != cudaSuccess)
          return set_error(BSP_ERR_ALLOC, "cudaHostAlloc of a batch slot failed");
        sl.h_bytes = tb;
      }
      std::vector<void*> ptrs;
      size_t o = 0;
      for (auto& pr : parts) {
        if (pr.second) memcpy(static_cast<uint8_t*>(sl.h) + o, pr.first, pr.second);
        ptrs.push_back(static_cast<uint8_t*>(sl.d) + o);
        o += align256(pr.second);
      }
      spmm_bind_tables(p, ptrs);
      p->d_blob = sl.d;
      if (sw) p->d_split_ws = reinterpret_cast<float*>(static_cast<uint8_t*>(sl.d) + tb);
      void* h_dev = nullptr;
      st = cuda_check(cudaHostGetDevicePointer(&h_dev, sl.h, 0), "cudaHostGetDevicePointer");
      if (st != BSP_OK) return st;
      fetch_mapped_words<<<static_cast<unsigned>(std::max(1, dev->sm_count)), 256, 0, sc>>>(
          static_cast<uint4*>(sl.d), static_cast<const uint4*>(h_dev), tb / 16);
      st = cuda_check(cudaGetLastError(), "plan table fetch");
      // 4. job k's kernel once its inputs are in; its C goes out while the
      //    later jobs' inputs still come in (the copies run both ways)
      const bsp_spmm_host_job& j = jobs[k];
      bsp_bsr_desc A{j.M, j.K, j.R, j.C, j.nnzb, d[k].rp, d[k].ci, d[k].val};
      const int64_t nh = j.N / panels[k];
      for (int h = 0; h < panels[k] && st == BSP_OK; ++h) {
        const size_t e = 4 * k + static_cast<size_t>(h);
        st = cuda_check(cudaStreamWaitEvent(sc, dev->ev_in[e], 0), "cudaStreamWaitEvent");
        if (st == BSP_OK) st = bsp_spmm_execute(p, &A, d[k].B + h * nh, j.N, d[k].C + h * nh, j.N, sc);
        if (st == BSP_OK) st = cuda_check(cudaEventRecord(dev->ev_out[e], sc), "cudaEventRecord");
        if (st == BSP_OK) st = cuda_check(cudaStreamWaitEvent(sd, dev->ev_out[e], 0), "cudaStreamWaitEvent");
        if (st != BSP_OK) break;
        if (panels[k] == 1) {
          st = cuda_check(cudaMemcpyAsync(j.C_out, d[k].C, sizeof(uint16_t) * j.M * j.N, cudaMemcpyDeviceToHost, sd),
                          "D2H C");
        } else {
          const size_t pitch = sizeof(uint16_t) * static_cast<size_t>(j.N), part = pitch / panels[k];
          st = cuda_check(cudaMemcpy2DAsync(reinterpret_cast<uint8_t*>(j.C_out) + h * part, pitch,
                                            reinterpret_cast<const uint8_t*>(d[k].C) + h * part, pitch, part,
                                            static_cast<size_t>(j.M), cudaMemcpyDeviceToHost, sd),
                          "D2H C panel");
        }
      }
    }
    if (st == BSP_OK) st = cuda_check(cudaStreamSynchronize(sd), "sync");
    if (st == BSP_OK) st = cuda_check(cudaStreamSynchronize(sc), "sync");
    return st;
  };
  s = run();
  join_upto(nj - 1);
  if (s != BSP_OK) {
    cudaStreamSynchronize(sh);
    cudaStreamSynchronize(sc);
    cudaStreamSynchronize(sd);
  }
  for (bsp_spmm_plan* p : plans) {
    if (p) p->blob_borrowed = true;  // tables live in the device's batch slots
    bsp_spmm_plan_destroy(p);
  }
  if (s != BSP_OK) return s;
  return bsp_device_synchronize(dev);
}

bsp_status bsp_spmm_host_profile(bsp_device* dev, int64_t M, int64_t K, int32_t R, int32_t C,
                                 int64_t nnzb, const int32_t* row_ptr, const int32_t* col_idx,
                                 const uint16_t* values, const uint16_t* B, int64_t N,
                                 uint16_t* C_out, bsp_strategy strategy, const bsp_spmm_opts* opts,
                                 int32_t iters, double* ms_per_launch) {
  if (iters < 1 || !ms_per_launch) return set_error(BSP_ERR_INVALID_ARG, "iters >= 1 and ms_per_launch required");
  return spmm_host_impl(dev, M, K, R, C, nnzb, row_ptr, col_idx, values, B, N, C_out, strategy,
                        opts, iters, ms_per_launch);
}

// --------------------------------------------------------------- SDDMM ----
static bsp_status sddmm_plan_create_impl(bsp_device* dev, const bsp_bsr_desc* mask,
                                         const int32_t* host_row_ptr, const int32_t* host_col_idx, int64_t K,
                                         bsp_strategy strategy, const bsp_sddmm_opts* opts, bool borrow,
                                         cudaStream_t stream, bsp_sddmm_plan** out);

bsp_status bsp_sddmm_plan_create(bsp_device* dev, const bsp_bsr_desc* mask,
                                 const int32_t* host_row_ptr, const int32_t* host_col_idx,
                                 int64_t K, bsp_strategy strategy, const bsp_sddmm_opts* opts,
                                 bsp_sddmm_plan** out) {
  return sddmm_plan_create_impl(dev, mask, host_row_ptr, host_col_idx, K, strategy, opts, false, nullptr,
                                out);
}

static bsp_status sddmm_plan_create_impl(bsp_device* dev, const bsp_bsr_desc* mask,
                                         const int32_t* host_row_ptr, const int32_t* host_col_idx, int64_t K,
                                         bsp_strategy strategy, const bsp_sddmm_opts* opts, bool borrow,
                                         cudaStream_t stream, bsp_sddmm_plan** out) {
  if (!dev || !out) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  bsp_status s = check_desc(mask, false);
  if (s != BSP_OK) return s;
  std::vector<int32_t> rp, ci;
  const int32_t *prp = nullptr, *pci = nullptr;
  s = host_pattern(mask, host_row_ptr, host_col_idx, &rp, &ci, &prp, &pci);
  if (s != BSP_OK) return s;
  bsp_sddmm_plan* p = new (std::nothrow) bsp_sddmm_plan();
  if (!p) return set_error(BSP_ERR_ALLOC, "host allocation failed");
  p->dev = dev;
  p->M = mask->rows;
  p->N = mask->cols;
  p->K = K;
  p->R = mask->R;
  p->C = mask->C;
  p->nnzb = mask->nnzb;
  p->strategy = strategy;
  s = plan_sddmm_host(p, prp, pci, dev->sm_count, dev->max_smem_optin, opts);
  if (s != BSP_OK) {
    delete p;
    return s;
  }
  std::vector<void*> ptrs;
  const std::vector<std::pair<const void*, size_t>> parts = {
      {p->h_units.data(), p->h_units.size() * sizeof(SddmmUnit)},
      {p->h_cta_begin.data(), p->h_cta_begin.size() * sizeof(int32_t)},
      {p->h_rs_units.data(), p->h_rs_units.size() * sizeof(SddmmRsUnit)}};
  s = borrow ? upload_blob_borrowed(dev, parts, stream, &p->d_blob, &p->blob_bytes, &ptrs)
             : upload_blob(parts, &p->d_blob, &p->blob_bytes, &ptrs);
  p->blob_borrowed = borrow;
  if (s != BSP_OK) {
    delete p;
    return s;
  }
  p->d_units = static_cast<SddmmUnit*>(ptrs[0]);
  p->d_cta_begin = static_cast<int32_t*>(ptrs[1]);
  p->d_rs_units = static_cast<SddmmRsUnit*>(ptrs[2]);
  *out = p;
  return BSP_OK;
}

bsp_status bsp_sddmm_execute(const bsp_sddmm_plan* plan, const bsp_bsr_desc* mask, const void* A,
                             int64_t lda, const void* B, int64_t ldb, void* out_values,
                             void* stream) {
  if (!plan || !A || !B || (!out_values && plan->nnzb > 0))
    return set_error(BSP_ERR_INVALID_ARG, "null argument");
  bsp_status s = check_desc(mask, false);
  if (s != BSP_OK) return s;
  if (mask->rows != plan->M || mask->cols != plan->N || mask->R != plan->R ||
      mask->C != plan->C || mask->nnzb != plan->nnzb)
    return set_error(BSP_ERR_INVALID_ARG, "mask does not match the plan's pattern");
  if (lda < plan->K || ldb < plan->N)
    return set_error(BSP_ERR_INVALID_ARG, "leading dimensions too small");
  if (reinterpret_cast<uintptr_t>(out_values) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "out_values must be 16-byte aligned");
  return launch_sddmm(plan, mask, A, lda, B, ldb, out_values, static_cast<cudaStream_t>(stream));
}

bsp_status bsp_sddmm_plan_destroy(bsp_sddmm_plan* plan) {
  if (!plan) return BSP_OK;
  if (plan->d_blob && !plan->blob_borrowed) cudaFree(plan->d_blob);
  delete plan;
  return BSP_OK;
}

bsp_status bsp_sddmm_plan_info(const bsp_sddmm_plan* p, int64_t info[16]) {
  if (!p || !info) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  memset(info, 0, sizeof(int64_t) * 16);
  info[0] = p->n_units;
  info[1] = p->grid;
  info[4] = p->Rs;
  info[5] = p->kc;
  info[6] = p->stages;
  info[7] = p->keep_a;
  info[8] = static_cast<int64_t>(p->blob_bytes);
  info[9] = p->smem_bytes;
  info[10] = p->tmem_cols;
  info[11] = p->variant;
  info[12] = static_cast<int64_t>((p->variant == 1 ? sizeof(SddmmRsUnit) : sizeof(SddmmUnit)) / 4);
  info[13] = p->nseg_max;
  info[14] = p->nprod;
  return BSP_OK;
}

bsp_status bsp_sddmm(bsp_device* dev, const bsp_bsr_desc* mask, const void* A, int64_t lda,
                     const void* B, int64_t ldb, int64_t K, void* out_values,
                     bsp_strategy strategy, const bsp_sddmm_opts* opts, void* stream) {
  bsp_sddmm_plan* p = nullptr;
  bsp_status s = bsp_sddmm_plan_create(dev, mask, nullptr, nullptr, K, strategy, opts, &p);
  if (s != BSP_OK) return s;
  s = bsp_sddmm_execute(p, mask, A, lda, B, ldb, out_values, stream);
  if (s == BSP_OK) s = cuda_check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "sync");
  bsp_sddmm_plan_destroy(p);
  if (s == BSP_OK) s = bsp_device_synchronize(dev);
  return s;
}

struct SddmmLaunchCtx {
  const bsp_sddmm_plan* p;
  const bsp_bsr_desc* mask;
  const void* A;
  const void* B;
  void* out;
  int64_t K, N;
  cudaStream_t stream;
};
static bsp_status sddmm_launch_ctx(const void* v) {
  const SddmmLaunchCtx* c = static_cast<const SddmmLaunchCtx*>(v);
  return bsp_sddmm_execute(c->p, c->mask, c->A, c->K, c->B, c->N, c->out, c->stream);
}

static bsp_status sddmm_host_impl(bsp_device* dev, int64_t M, int64_t N, int32_t R, int32_t C,
                                  int64_t nnzb, const int32_t* row_ptr, const int32_t* col_idx,
                                  const uint16_t* mask_values, const uint16_t* A, const uint16_t* B,
                                  int64_t K, uint16_t* out_values, bsp_strategy strategy,
                                  const bsp_sddmm_opts* opts, int32_t iters, double* ms_out) {
  if (!dev || !row_ptr || !A || !B || (nnzb > 0 && (!col_idx || !out_values)))
    return set_error(BSP_ERR_INVALID_ARG, "null argument");
  if (R <= 0 || C <= 0 || M % R || N % C) return set_error(BSP_ERR_INVALID_ARG, "bad dimensions");
  const int64_t nbr = M / R;
  const size_t blk = sizeof(uint16_t) * nnzb * R * C;
  const size_t b_mask = mask_values ? align256(blk) : 0;
  const size_t b_out = align256(std::max<size_t>(blk, 16));
  const size_t b_rp = align256(sizeof(int32_t) * (nbr + 1));
  const size_t b_ci = align256(sizeof(int32_t) * std::max<int64_t>(nnzb, 1));
  const size_t b_A = align256(sizeof(uint16_t) * M * K);
  const size_t b_B = align256(sizeof(uint16_t) * K * N);
  bsp_status s = ws_reserve(dev, b_mask + b_out + b_rp + b_ci + b_A + b_B);
  if (s != BSP_OK) return s;
  uint8_t* w = static_cast<uint8_t*>(dev->ws);
  void* d_out = w;
  void* d_mask = mask_values ? w + b_out : nullptr;
  int32_t* d_rp = reinterpret_cast<int32_t*>(w + b_out + b_mask);
  int32_t* d_ci = reinterpret_cast<int32_t*>(w + b_out + b_mask + b_rp);
  void* d_A = w + b_out + b_mask + b_rp + b_ci;
  void* d_B = w + b_out + b_mask + b_rp + b_ci + b_A;
  if ((s = host_streams(dev, 1)) != BSP_OK) return s;
  cudaStream_t stream = dev->s_comp;
  struct SyncOnExit {  // nothing of this call may still run when the workspace is reused
    cudaStream_t st;
    ~SyncOnExit() { cudaStreamSynchronize(st); }
  } sync_on_exit{stream};
  if ((s = cuda_check(cudaMemcpyAsync(d_A, A, sizeof(uint16_t) * M * K, cudaMemcpyHostToDevice, stream), "H2D A")) != BSP_OK) return s;
  if ((s = cuda_check(cudaMemcpyAsync(d_B, B, sizeof(uint16_t) * K * N, cudaMemcpyHostToDevice, stream), "H2D B")) != BSP_OK) return s;
  if ((s = cuda_check(cudaMemcpyAsync(d_rp, row_ptr, sizeof(int32_t) * (nbr + 1), cudaMemcpyHostToDevice, stream), "H2D row_ptr")) != BSP_OK) return s;
  if (nnzb > 0) {
    if ((s = cuda_check(cudaMemcpyAsync(d_ci, col_idx, sizeof(int32_t) * nnzb, cudaMemcpyHostToDevice, stream), "H2D col_idx")) != BSP_OK) return s;
    if (mask_values &&
        (s = cuda_check(cudaMemcpyAsync(d_mask, mask_values, blk, cudaMemcpyHostToDevice, stream), "H2D mask")) != BSP_OK)
      return s;
  }
  bsp_bsr_desc mask{M, N, R, C, nnzb, d_rp, d_ci, d_mask};
  bsp_sddmm_plan* p = nullptr;
  s = sddmm_plan_create_impl(dev, &mask, row_ptr, col_idx, K, strategy, opts, true, stream, &p);
  if (s != BSP_OK) return s;
  s = bsp_sddmm_execute(p, &mask, d_A, K, d_B, N, d_out, stream);
  if (s == BSP_OK && iters > 0) {
    const SddmmLaunchCtx ctx{p, &mask, d_A, d_B, d_out, K, N, stream};
    s = time_launches(iters, ms_out, stream, sddmm_launch_ctx, &ctx);
  }
  if (s == BSP_OK && nnzb > 0)
    s = cuda_check(cudaMemcpyAsync(out_values, d_out, blk, cudaMemcpyDeviceToHost, stream), "D2H out");
  if (s == BSP_OK) s = cuda_check(cudaStreamSynchronize(stream), "sync");
  bsp_sddmm_plan_destroy(p);
  if (s == BSP_OK) s = bsp_device_synchronize(dev);
  return s;
}

bsp_status bsp_sddmm_host(bsp_device* dev, int64_t M, int64_t N, int32_t R, int32_t C,
                          int64_t nnzb, const int32_t* row_ptr, const int32_t* col_idx,
                          const uint16_t* mask_values, const uint16_t* A, const uint16_t* B,
                          int64_t K, uint16_t* out_values, bsp_strategy strategy,
                          const bsp_sddmm_opts* opts) {
  return sddmm_host_impl(dev, M, N, R, C, nnzb, row_ptr, col_idx, mask_values, A, B, K,
                         out_values, strategy, opts, 0, nullptr);
}

bsp_status bsp_sddmm_host_profile(bsp_device* dev, int64_t M, int64_t N, int32_t R, int32_t C,
                                  int64_t nnzb, const int32_t* row_ptr, const int32_t* col_idx,
                                  const uint16_t* mask_values, const uint16_t* A,
                                  const uint16_t* B, int64_t K, uint16_t* out_values,
                                  bsp_strategy strategy, const bsp_sddmm_opts* opts, int32_t iters,
                                  double* ms_per_launch) {
  if (iters < 1 || !ms_per_launch) return set_error(BSP_ERR_INVALID_ARG, "iters >= 1 and ms_per_launch required");
  return sddmm_host_impl(dev, M, N, R, C, nnzb, row_ptr, col_idx, mask_values, A, B, K,
                         out_values, strategy, opts, iters, ms_per_launch);
}

// -------------------------------------------------------------- SpGEMM ----
static bsp_status spgemm_check_pair(const bsp_bsr_desc* A, const bsp_bsr_desc* B) {
  if (A->cols != B->rows || A->C != B->R)
    return set_error(BSP_ERR_INVALID_ARG, "A's columns (and block width) must match B's rows");
  return BSP_OK;
}

static bsp_status spgemm_plan_create_impl(bsp_device* dev, const bsp_bsr_desc* A,
                                          const int32_t* a_host_row_ptr, const int32_t* a_host_col_idx,
                                          const bsp_bsr_desc* B, const int32_t* b_host_row_ptr,
                                          const int32_t* b_host_col_idx, const bsp_spmm_opts* opts,
                                          bool borrow, cudaStream_t stream, bsp_spgemm_plan** out);

bsp_status bsp_spgemm_plan_create(bsp_device* dev, const bsp_bsr_desc* A,
                                  const int32_t* a_host_row_ptr, const int32_t* a_host_col_idx,
                                  const bsp_bsr_desc* B, const int32_t* b_host_row_ptr,
                                  const int32_t* b_host_col_idx, const bsp_spmm_opts* opts,
                                  bsp_spgemm_plan** out) {
  return spgemm_plan_create_impl(dev, A, a_host_row_ptr, a_host_col_idx, B, b_host_row_ptr, b_host_col_idx,
                                 opts, false, nullptr, out);
}

static bsp_status spgemm_plan_create_impl(bsp_device* dev, const bsp_bsr_desc* A,
                                          const int32_t* a_host_row_ptr, const int32_t* a_host_col_idx,
                                          const bsp_bsr_desc* B, const int32_t* b_host_row_ptr,
                                          const int32_t* b_host_col_idx, const bsp_spmm_opts* opts,
                                          bool borrow, cudaStream_t stream, bsp_spgemm_plan** out) {
  if (!dev || !out) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  bsp_status s = check_desc(A, false);
  if (s == BSP_OK) s = check_desc(B, false);
  if (s == BSP_OK) s = spgemm_check_pair(A, B);
  if (s != BSP_OK) return s;
  std::vector<int32_t> arp, aci, brp, bci;
  const int32_t *parp = nullptr, *paci = nullptr, *pbrp = nullptr, *pbci = nullptr;
  s = host_pattern(A, a_host_row_ptr, a_host_col_idx, &arp, &aci, &parp, &paci);
  if (s == BSP_OK) s = host_pattern(B, b_host_row_ptr, b_host_col_idx, &brp, &bci, &pbrp, &pbci);
  if (s != BSP_OK) return s;
  bsp_spgemm_plan* p = new (std::nothrow) bsp_spgemm_plan();
  if (!p) return set_error(BSP_ERR_ALLOC, "host allocation failed");
  p->dev = dev;
  p->M = A->rows;
  p->K = A->cols;
  p->N = B->cols;
  p->Ra = A->R;
  p->Ca = A->C;
  p->Cb = B->C;
  p->nnzb_a = A->nnzb;
  p->nnzb_b = B->nnzb;
  s = plan_spgemm_host(p, parp, paci, pbrp, pbci, dev->sm_count, dev->max_smem_optin, opts);
  if (s != BSP_OK) {
    delete p;
    return s;
  }
  std::vector<void*> ptrs;
  const std::vector<std::pair<const void*, size_t>> parts = {
      {p->h_units.data(), p->h_units.size() * sizeof(SpgemmUnit)},
      {p->h_steps.data(), p->h_steps.size() * sizeof(SpgemmStep)},
      {p->h_cta_begin.data(), p->h_cta_begin.size() * sizeof(int32_t)}};
  s = borrow ? upload_blob_borrowed(dev, parts, stream, &p->d_blob, &p->blob_bytes, &ptrs)
             : upload_blob(parts, &p->d_blob, &p->blob_bytes, &ptrs);
  p->blob_borrowed = borrow;
  if (s != BSP_OK) {
    delete p;
    return s;
  }
  p->d_units = static_cast<SpgemmUnit*>(ptrs[0]);
  p->d_steps = static_cast<SpgemmStep*>(ptrs[1]);
  p->d_cta_begin = static_cast<int32_t*>(ptrs[2]);
  *out = p;
  return BSP_OK;
}

bsp_status bsp_spgemm_pattern(const bsp_spgemm_plan* p, int64_t* nnzb_out, int32_t* row_ptr_out,
                              int32_t* col_idx_out) {
  if (!p || !nnzb_out) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  *nnzb_out = static_cast<int64_t>(p->out_col_idx.size());
  if (row_ptr_out) memcpy(row_ptr_out, p->out_row_ptr.data(), p->out_row_ptr.size() * sizeof(int32_t));
  if (col_idx_out && !p->out_col_idx.empty())
    memcpy(col_idx_out, p->out_col_idx.data(), p->out_col_idx.size() * sizeof(int32_t));
  return BSP_OK;
}

bsp_status bsp_spgemm_execute(const bsp_spgemm_plan* plan, const bsp_bsr_desc* A,
                              const bsp_bsr_desc* B, void* out_values, void* stream) {
  if (!plan) return set_error(BSP_ERR_INVALID_ARG, "null plan");
  bsp_status s = check_desc(A, true);
  if (s == BSP_OK) s = check_desc(B, true);
  if (s == BSP_OK) s = spgemm_check_pair(A, B);
  if (s != BSP_OK) return s;
  if (A->rows != plan->M || A->cols != plan->K || B->cols != plan->N || A->R != plan->Ra ||
      A->C != plan->Ca || B->C != plan->Cb || A->nnzb != plan->nnzb_a || B->nnzb != plan->nnzb_b)
    return set_error(BSP_ERR_INVALID_ARG, "A or B does not match the plan's patterns");
  if (!plan->out_col_idx.empty() && !out_values)
    return set_error(BSP_ERR_INVALID_ARG, "out_values missing");
  return launch_spgemm(plan, A->values, B->values, out_values, static_cast<cudaStream_t>(stream));
}

bsp_status bsp_spgemm_plan_destroy(bsp_spgemm_plan* plan) {
  if (!plan) return BSP_OK;
  if (plan->d_blob && !plan->blob_borrowed) cudaFree(plan->d_blob);
  delete plan;
  return BSP_OK;
}

bsp_status bsp_spgemm_plan_info(const bsp_spgemm_plan* p, int64_t info[16]) {
  if (!p || !info) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  memset(info, 0, sizeof(int64_t) * 16);
  info[0] = p->n_units;
  info[1] = p->grid;
  info[2] = p->n_steps;
  info[3] = p->pairs;
  info[4] = static_cast<int64_t>(p->out_col_idx.size());
  info[5] = p->kc;
  info[6] = p->stages;
  info[7] = p->sps;
  info[8] = static_cast<int64_t>(p->blob_bytes);
  info[9] = p->smem_bytes;
  info[10] = p->tmem_cols;
  info[11] = p->nseg_max;
  info[12] = p->nprod;
  info[13] = p->n_boxes;
  return BSP_OK;
}

struct SpgemmLaunchCtx {
  const bsp_spgemm_plan* p;
  const bsp_bsr_desc* A;
  const bsp_bsr_desc* B;
  void* out;
  cudaStream_t stream;
};
static bsp_status spgemm_launch_ctx(const void* v) {
  const SpgemmLaunchCtx* c = static_cast<const SpgemmLaunchCtx*>(v);
  return bsp_spgemm_execute(c->p, c->A, c->B, c->out, c->stream);
}

bsp_status bsp_spgemm_host(bsp_device* dev, int64_t M, int64_t K, int64_t N, int32_t Ra, int32_t Ca,
                           int32_t Cb, int64_t a_nnzb, const int32_t* a_row_ptr,
                           const int32_t* a_col_idx, const uint16_t* a_values, int64_t b_nnzb,
                           const int32_t* b_row_ptr, const int32_t* b_col_idx,
                           const uint16_t* b_values, int64_t out_cap, int64_t* out_nnzb,
                           int32_t* out_row_ptr, int32_t* out_col_idx, uint16_t* out_values,
                           const bsp_spmm_opts* opts, int32_t iters, double* ms_per_launch) {
  if (!dev || !a_row_ptr || !b_row_ptr || !out_nnzb || (a_nnzb > 0 && (!a_col_idx || !a_values)) ||
      (b_nnzb > 0 && (!b_col_idx || !b_values)) || (iters > 0 && !ms_per_launch) || iters < 0)
    return set_error(BSP_ERR_INVALID_ARG, "null argument");
  if (Ra <= 0 || Ca <= 0 || Cb <= 0 || M <= 0 || K <= 0 || N <= 0 || M % Ra || K % Ca || N % Cb)
    return set_error(BSP_ERR_INVALID_ARG, "bad dimensions");
  const int64_t nbr = M / Ra, nbk = K / Ca;
  // planning needs only the patterns; the device copies come after the size query
  bsp_spgemm_plan probe;
  probe.dev = dev;
  probe.M = M;
  probe.K = K;
  probe.N = N;
  probe.Ra = Ra;
  probe.Ca = Ca;
  probe.Cb = Cb;
  probe.nnzb_a = a_nnzb;
  probe.nnzb_b = b_nnzb;
  const bool query = out_values == nullptr;
  bsp_status s = BSP_OK;
  bsp_spgemm_plan* p = nullptr;
  if (query) {
    s = plan_spgemm_host(&probe, a_row_ptr, a_col_idx, b_row_ptr, b_col_idx, dev->sm_count,
                         dev->max_smem_optin, opts);
    if (s == BSP_OK) *out_nnzb = static_cast<int64_t>(probe.out_col_idx.size());
    return s;
  }
  if (!out_row_ptr || (out_cap > 0 && !out_col_idx))
    return set_error(BSP_ERR_INVALID_ARG, "output arrays missing");
  const size_t a_blk = sizeof(uint16_t) * a_nnzb * Ra * Ca;
  const size_t b_blk = sizeof(uint16_t) * b_nnzb * Ca * Cb;
  const size_t o_cap = sizeof(uint16_t) * std::max<int64_t>(out_cap, 0) * Ra * Cb;
  const size_t b_av = align256(std::max<size_t>(a_blk, 16)), b_bv = align256(std::max<size_t>(b_blk, 16));
  const size_t b_ov = align256(std::max<size_t>(o_cap, 16));
  const size_t b_arp = align256(sizeof(int32_t) * (nbr + 1)), b_aci = align256(sizeof(int32_t) * std::max<int64_t>(a_nnzb, 1));
  const size_t b_brp = align256(sizeof(int32_t) * (nbk + 1)), b_bci = align256(sizeof(int32_t) * std::max<int64_t>(b_nnzb, 1));
  s = ws_reserve(dev, b_av + b_bv + b_ov + b_arp + b_aci + b_brp + b_bci);
  if (s != BSP_OK) return s;
  uint8_t* w = static_cast<uint8_t*>(dev->ws);
  void* d_av = w;
  void* d_bv = w + b_av;
  void* d_ov = w + b_av + b_bv;
  int32_t* d_arp = reinterpret_cast<int32_t*>(w + b_av + b_bv + b_ov);
  int32_t* d_aci = reinterpret_cast<int32_t*>(w + b_av + b_bv + b_ov + b_arp);
  int32_t* d_brp = reinterpret_cast<int32_t*>(w + b_av + b_bv + b_ov + b_arp + b_aci);
  int32_t* d_bci = reinterpret_cast<int32_t*>(w + b_av + b_bv + b_ov + b_arp + b_aci + b_brp);
  if ((s = host_streams(dev, 1)) != BSP_OK) return s;
  cudaStream_t stream = dev->s_comp;
  struct SyncOnExit {  // nothing of this call may still run when the workspace is reused
    cudaStream_t st;
    ~SyncOnExit() { cudaStreamSynchronize(st); }
  } sync_on_exit{stream};
  struct Cp { void* d; const void* h; size_t n; const char* what; };
  const Cp cps[] = {{d_av, a_values, a_blk, "H2D A values"}, {d_bv, b_values, b_blk, "H2D B values"},
                    {d_arp, a_row_ptr, sizeof(int32_t) * (nbr + 1), "H2D A row_ptr"},
                    {d_aci, a_col_idx, sizeof(int32_t) * a_nnzb, "H2D A col_idx"},
                    {d_brp, b_row_ptr, sizeof(int32_t) * (nbk + 1), "H2D B row_ptr"},
                    {d_bci, b_col_idx, sizeof(int32_t) * b_nnzb, "H2D B col_idx"}};
  for (const Cp& c : cps)
    if (c.n > 0 && (s = cuda_check(cudaMemcpyAsync(c.d, c.h, c.n, cudaMemcpyHostToDevice, stream), c.what)) != BSP_OK)
      return s;
  const bsp_bsr_desc A{M, K, Ra, Ca, a_nnzb, d_arp, d_aci, d_av};
  const bsp_bsr_desc B{K, N, Ca, Cb, b_nnzb, d_brp, d_bci, d_bv};
  s = spgemm_plan_create_impl(dev, &A, a_row_ptr, a_col_idx, &B, b_row_ptr, b_col_idx, opts, true, stream, &p);
  if (s != BSP_OK) return s;
  const int64_t n_out = static_cast<int64_t>(p->out_col_idx.size());
  *out_nnzb = n_out;
  if (n_out > out_cap) {
    bsp_spgemm_plan_destroy(p);
    return set_error(BSP_ERR_INVALID_ARG, "out_cap is smaller than the product's block count");
  }
  s = bsp_spgemm_execute(p, &A, &B, d_ov, stream);
  if (s == BSP_OK && iters > 0) {
    const SpgemmLaunchCtx ctx{p, &A, &B, d_ov, stream};
    s = time_launches(iters, ms_per_launch, stream, spgemm_launch_ctx, &ctx);
  }
  if (s == BSP_OK && n_out > 0)
    s = cuda_check(cudaMemcpyAsync(out_values, d_ov, sizeof(uint16_t) * n_out * Ra * Cb,
                                   cudaMemcpyDeviceToHost, stream),
                   "D2H C values");
  if (s == BSP_OK) s = cuda_check(cudaStreamSynchronize(stream), "sync");
  if (s == BSP_OK) {
    memcpy(out_row_ptr, p->out_row_ptr.data(), p->out_row_ptr.size() * sizeof(int32_t));
    if (n_out > 0) memcpy(out_col_idx, p->out_col_idx.data(), n_out * sizeof(int32_t));
  }
  bsp_spgemm_plan_destroy(p);
  if (s == BSP_OK) s = bsp_device_synchronize(dev);
  return s;
}

// ----------------------------------------------------------- attention ----
static bsp_status attn_plan_create_impl(bsp_device* dev, const bsp_bsr_desc* mask,
                                        const int32_t* host_row_ptr, const int32_t* host_col_idx, int64_t d,
                                        const bsp_spmm_opts* opts, bool borrow, cudaStream_t stream,
                                        bsp_attn_plan** out);

bsp_status bsp_attn_plan_create(bsp_device* dev, const bsp_bsr_desc* mask, const int32_t* host_row_ptr,
                                const int32_t* host_col_idx, int64_t d, const bsp_spmm_opts* opts,
                                bsp_attn_plan** out) {
  return attn_plan_create_impl(dev, mask, host_row_ptr, host_col_idx, d, opts, false, nullptr, out);
}

static bsp_status attn_plan_create_impl(bsp_device* dev, const bsp_bsr_desc* mask,
                                        const int32_t* host_row_ptr, const int32_t* host_col_idx, int64_t d,
                                        const bsp_spmm_opts* opts, bool borrow, cudaStream_t stream,
                                        bsp_attn_plan** out) {
  if (!dev || !out) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  bsp_status s = check_desc(mask, false);
  if (s != BSP_OK) return s;
  if (mask->R != 32 || mask->C != 32 || mask->rows != mask->cols)
    return set_error(BSP_ERR_INVALID_ARG, "attention mask must be square with 32 x 32 blocks");
  std::vector<int32_t> rp, ci;
  const int32_t *prp = nullptr, *pci = nullptr;
  s = host_pattern(mask, host_row_ptr, host_col_idx, &rp, &ci, &prp, &pci);
  if (s != BSP_OK) return s;
  bsp_attn_plan* p = new (std::nothrow) bsp_attn_plan();
  if (!p) return set_error(BSP_ERR_ALLOC, "host allocation failed");
  p->dev = dev;
  p->S = mask->rows;
  p->d = d;
  p->nnzb = mask->nnzb;
  s = plan_attn_host(p, prp, pci, dev->sm_count, dev->max_smem_optin, opts);
  if (s != BSP_OK) {
    delete p;
    return s;
  }
  std::vector<void*> ptrs;
  // split-unit counters: two sets, used by alternate launches (each launch zeroes the other)
  const std::vector<int32_t> zeros(2 * static_cast<size_t>(p->n_counters), 0);
  const std::vector<std::pair<const void*, size_t>> parts = {
      {p->h_units.data(), p->h_units.size() * sizeof(AttnUnit)},
      {p->h_chunks.data(), p->h_chunks.size() * sizeof(AttnChunk)},
      {p->h_cta_begin.data(), p->h_cta_begin.size() * sizeof(int32_t)},
      {zeros.data(), zeros.size() * sizeof(int32_t)}};
  s = borrow ? upload_blob_borrowed(dev, parts, stream, &p->d_blob, &p->blob_bytes, &ptrs)
             : upload_blob(parts, &p->d_blob, &p->blob_bytes, &ptrs);
  p->blob_borrowed = borrow;
  if (s != BSP_OK) {
    delete p;
    return s;
  }
  p->d_units = static_cast<AttnUnit*>(ptrs[0]);
  p->d_chunks = static_cast<AttnChunk*>(ptrs[1]);
  p->d_cta_begin = static_cast<int32_t*>(ptrs[2]);
  p->d_counters = static_cast<int32_t*>(ptrs[3]);
  if (p->n_slots > 0) {
    const size_t wb = sizeof(float) * 128 * (p->d + 2) * p->n_slots;
    if (borrow) {
      if (dev->aux_ws_bytes < wb) {
        if (dev->aux_ws) cudaFree(dev->aux_ws);
        dev->aux_ws = nullptr;
        dev->aux_ws_bytes = 0;
        if (cudaMalloc(&dev->aux_ws, wb) != cudaSuccess) {
          bsp_attn_plan_destroy(p);
          return set_error(BSP_ERR_ALLOC, "cudaMalloc of the attention merge workspace failed");
        }
        dev->aux_ws_bytes = wb;
      }
      p->d_work = static_cast<float*>(dev->aux_ws);
    } else if (cudaMalloc(&p->d_work, wb) != cudaSuccess) {
      bsp_attn_plan_destroy(p);
      return set_error(BSP_ERR_ALLOC, "cudaMalloc of the attention merge workspace failed");
    }
  }
  *out = p;
  return BSP_OK;
}

bsp_status bsp_attn_execute(const bsp_attn_plan* plan, const void* Q, int64_t ldq, const void* K,
                            int64_t ldk, const void* V, int64_t ldv, float scale, void* O,
                            int64_t ldo, void* stream) {
  if (!plan || !Q || !K || !V || !O) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  if (ldq < plan->d || ldk < plan->d || ldv < plan->d || ldo < plan->d)
    return set_error(BSP_ERR_INVALID_ARG, "leading dimensions must be >= d");
  return launch_attn(plan, Q, ldq, K, ldk, V, ldv, scale, O, ldo, static_cast<cudaStream_t>(stream));
}

bsp_status bsp_attn_plan_destroy(bsp_attn_plan* plan) {
  if (!plan) return BSP_OK;
  if (plan->d_blob && !plan->blob_borrowed) cudaFree(plan->d_blob);
  if (plan->d_work && !plan->blob_borrowed) cudaFree(plan->d_work);
  delete plan;
  return BSP_OK;
}

bsp_status bsp_attn_plan_info(const bsp_attn_plan* p, int64_t info[16]) {
  if (!p || !info) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  memset(info, 0, sizeof(int64_t) * 16);
  info[0] = p->n_units;
  info[1] = p->grid;
  info[2] = p->n_chunks;
  info[3] = p->mask_blocks;
  info[4] = p->S;
  info[5] = p->d;
  info[6] = p->n_slots;
  info[7] = p->n_counters;
  info[8] = static_cast<int64_t>(p->blob_bytes);
  info[9] = p->smem_bytes;
  info[10] = p->tmem_cols;
  return BSP_OK;
}

bsp_status bsp_attn_host(bsp_device* dev, int64_t S, int64_t d, int64_t nnzb, const int32_t* row_ptr,
                         const int32_t* col_idx, const uint16_t* Q, const uint16_t* K,
                         const uint16_t* V, float scale, uint16_t* O, const bsp_spmm_opts* opts) {
  if (!dev || !row_ptr || !Q || !K || !V || !O || (nnzb > 0 && !col_idx))
    return set_error(BSP_ERR_INVALID_ARG, "null argument");
  if (S <= 0 || S % 32 || d <= 0) return set_error(BSP_ERR_INVALID_ARG, "bad dimensions");
  const int64_t nbr = S / 32;
  const size_t mat = sizeof(uint16_t) * S * d;
  const size_t b_m = align256(mat);
  const size_t b_rp = align256(sizeof(int32_t) * (nbr + 1));
  const size_t b_ci = align256(sizeof(int32_t) * std::max<int64_t>(nnzb, 1));
  bsp_status s = ws_reserve(dev, 4 * b_m + b_rp + b_ci);
  if (s != BSP_OK) return s;
  uint8_t* w = static_cast<uint8_t*>(dev->ws);
  void *dQ = w, *dK = w + b_m, *dV = w + 2 * b_m, *dO = w + 3 * b_m;
  int32_t* d_rp = reinterpret_cast<int32_t*>(w + 4 * b_m);
  int32_t* d_ci = reinterpret_cast<int32_t*>(w + 4 * b_m + b_rp);
  if ((s = host_streams(dev, 1)) != BSP_OK) return s;
  cudaStream_t stream = dev->s_comp;
  struct SyncOnExit {  // nothing of this call may still run when the workspace is reused
    cudaStream_t st;
    ~SyncOnExit() { cudaStreamSynchronize(st); }
  } sync_on_exit{stream};
  struct Cp { void* d; const void* h; size_t n; const char* what; };
  const Cp cps[] = {{dQ, Q, mat, "H2D Q"}, {dK, K, mat, "H2D K"}, {dV, V, mat, "H2D V"},
                    {d_rp, row_ptr, sizeof(int32_t) * (nbr + 1), "H2D row_ptr"},
                    {d_ci, col_idx, sizeof(int32_t) * nnzb, "H2D col_idx"}};
  for (const Cp& c : cps)
    if (c.n > 0 && (s = cuda_check(cudaMemcpyAsync(c.d, c.h, c.n, cudaMemcpyHostToDevice, stream), c.what)) != BSP_OK)
      return s;
  const bsp_bsr_desc mask{S, S, 32, 32, nnzb, d_rp, d_ci, nullptr};
  bsp_attn_plan* p = nullptr;
  s = attn_plan_create_impl(dev, &mask, row_ptr, col_idx, d, opts, true, stream, &p);
  if (s != BSP_OK) return s;
  s = bsp_attn_execute(p, dQ, d, dK, d, dV, d, scale, dO, d, stream);
  if (s == BSP_OK) s = cuda_check(cudaMemcpyAsync(O, dO, mat, cudaMemcpyDeviceToHost, stream), "D2H O");
  if (s == BSP_OK) s = cuda_check(cudaStreamSynchronize(stream), "sync");
  bsp_attn_plan_destroy(p);
  if (s == BSP_OK) s = bsp_device_synchronize(dev);
  return s;
}

// ----------------------------------------------------------- helpers ----
bsp_status bsp_partition_rows(const int32_t* row_ptr, int64_t n_block_rows, int32_t parts,
                              int64_t* bounds) {
  if (!row_ptr || !bounds || parts < 1 || n_block_rows < 0)
    return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  // Balance blocks plus one unit per row (every row costs its C writes).  The
  // ranges minimise the heaviest range (a row of a thousand blocks next to a
  // cut otherwise lands whole on one range), and among those that reach the
  // minimum, each range takes about its share of what is left.
  const int64_t n = n_block_rows;
  auto wt = [&](int64_t i) { return int64_t(row_ptr[i + 1]) - row_ptr[i] + 1; };
  const int64_t total = int64_t(row_ptr[n]) - row_ptr[0] + n;
  int64_t lo = 0, hi = std::max<int64_t>(total, 1);
  for (int64_t i = 0; i < n; ++i) lo = std::max(lo, wt(i));
  auto ranges_needed = [&](int64_t cap) {
    int64_t cnt = 0, w = 0;
    for (int64_t i = 0; i < n; ++i) {
      if (w + wt(i) > cap) {
        ++cnt;
        w = 0;
      }
      w += wt(i);
    }
    return cnt + (w > 0 ? 1 : 0);
  };
  while (lo < hi) {
    const int64_t mid = lo + (hi - lo) / 2;
    if (ranges_needed(mid) <= parts) hi = mid;
    else lo = mid + 1;
  }
  const int64_t cap = lo;
  // need[i]: ranges that rows [i, n) take at the cap (greedy, two pointers)
  std::vector<int64_t> need(static_cast<size_t>(n) + 1, 0);
  {
    int64_t j = n, w = 0;
    for (int64_t i = n - 1; i >= 0; --i) {
      w += wt(i);
      while (w > cap) {
        --j;
        w -= wt(j);
      }
      need[static_cast<size_t>(i)] = 1 + need[static_cast<size_t>(j)];
    }
  }
  bounds[0] = 0;
  int64_t r = 0, left = total;
  for (int p = 0; p + 1 < parts; ++p) {
    const int64_t share = left / (parts - p);
    int64_t w = 0;
    while (r < n && w + wt(r) <= cap &&
           (need[static_cast<size_t>(r)] > parts - p - 1 || 2 * (w + wt(r)) <= 2 * share + wt(r))) {
      w += wt(r);
      ++r;
    }
    left -= w;
    bounds[p + 1] = r;
  }
  bounds[parts] = n;
  return BSP_OK;
}

bsp_status bsp_serpentine_assign(int64_t n, int32_t parts, int32_t* owner, int32_t* slot) {
  if (n < 0 || parts < 1 || (n > 0 && (!owner || !slot)))
    return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  // weights n-1 .. 0 make the heaviest-first permutation the identity
  std::vector<int64_t> w(n);
  for (int64_t i = 0; i < n; ++i) w[i] = n - i;
  std::vector<std::vector<int32_t>> per;
  serpentine_order(w, parts, &per);
  for (int p = 0; p < parts; ++p)
    for (size_t k = 0; k < per[p].size(); ++k) {
      owner[per[p][k]] = p;
      slot[per[p][k]] = static_cast<int32_t>(k);
    }
  return BSP_OK;
}

}  // extern "C"

// ------------------------------------------------ host-only inspection ----
#include "bsp_testing.h"

extern "C" {

bsp_status bsp_testing_spmm_counters(const bsp_spmm_plan* plan, void** counters, int64_t* per_set,
                                     int32_t* next_set) {
  if (!plan || !counters || !per_set || !next_set) return set_error(BSP_ERR_INVALID_ARG, "null argument");
  *counters = plan->n_split_slots > 0 ? plan->d_split_counters : nullptr;
  *per_set = plan->n_split_slots;
  *next_set = static_cast<int32_t>(plan->launch_parity & 1u);
  return BSP_OK;
}

bsp_status bsp_testing_spmm_drop_stage(bsp_spmm_plan* plan, int32_t stage_plus_one) {
  if (!plan || stage_plus_one < 0) return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  if (plan->variant != 1)
    return set_error(BSP_ERR_UNSUPPORTED, "stage dropping is built into the row-stacked kernel only");
  plan->debug_drop_stage = stage_plus_one;
  return BSP_OK;
}

bsp_status bsp_spmm_plan_inspect(int64_t M, int64_t K, int32_t R, int32_t C, int64_t nnzb,
                                 const int32_t* row_ptr, const int32_t* col_idx, int64_t N,
                                 bsp_dtype c_type, bsp_strategy strategy,
                                 const bsp_spmm_opts* opts, int32_t sm_count, int32_t max_smem,
                                 int64_t info[16], int32_t* units_out, int32_t* cta_begin_out,
                                 int32_t* steps_out, int32_t* stage_list_out,
                                 int32_t* cta_stage_begin_out) {
  if (!row_ptr || !info || (nnzb > 0 && !col_idx) || R <= 0 || C <= 0)
    return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  bsp_spmm_plan p;
  p.M = M;
  p.K = K;
  p.N = N;
  p.R = R;
  p.C = C;
  p.nnzb = nnzb;
  p.c_type = c_type;
  p.strategy = strategy;
  bsp_status s = plan_spmm_host(&p, row_ptr, col_idx, sm_count, max_smem, opts);
  if (s != BSP_OK) return s;
  bsp_spmm_plan_info(&p, info);
  if (units_out) memcpy(units_out, p.h_units.data(), p.h_units.size() * sizeof(SpmmUnit));
  if (cta_begin_out)
    memcpy(cta_begin_out, p.h_cta_begin.data(), p.h_cta_begin.size() * sizeof(int32_t));
  if (steps_out) memcpy(steps_out, p.h_steps.data(), p.n_steps * p.step_stride * sizeof(int32_t));
  info[13] = static_cast<int64_t>(p.h_stage_list.size() / kRsStageWords);
  info[14] = p.nsub;
  if (stage_list_out && !p.h_stage_list.empty())
    memcpy(stage_list_out, p.h_stage_list.data(), p.h_stage_list.size() * sizeof(int32_t));
  if (cta_stage_begin_out && !p.h_cta_stage_begin.empty())
    memcpy(cta_stage_begin_out, p.h_cta_stage_begin.data(), p.h_cta_stage_begin.size() * sizeof(int32_t));
  return BSP_OK;
}

bsp_status bsp_spmm_plan_traffic(int64_t M, int64_t K, int32_t R, int32_t C, int64_t nnzb,
                                 const int32_t* row_ptr, const int32_t* col_idx, int64_t N,
                                 bsp_strategy strategy, const bsp_spmm_opts* opts, int32_t sm_count,
                                 int32_t max_smem, int64_t info[16], int64_t traffic[4]) {
  if (!row_ptr || !info || !traffic || (nnzb > 0 && !col_idx) || R <= 0 || C <= 0)
    return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  bsp_spmm_plan p;
  p.M = M;
  p.K = K;
  p.N = N;
  p.R = R;
  p.C = C;
  p.nnzb = nnzb;
  p.strategy = strategy;
  bsp_status s = plan_spmm_host(&p, row_ptr, col_idx, sm_count, max_smem, opts);
  if (s != BSP_OK) return s;
  bsp_spmm_plan_info(&p, info);
  spmm_plan_traffic(p, traffic);
  return BSP_OK;
}

bsp_status bsp_spmm_plan_entry_rows(int64_t M, int64_t K, int32_t R, int32_t C, int64_t nnzb,
                                    const int32_t* row_ptr, const int32_t* col_idx, int64_t N,
                                    bsp_strategy strategy, const bsp_spmm_opts* opts, int32_t sm_count,
                                    int32_t max_smem, int32_t* rows_out, int64_t* n_out) {
  if (!row_ptr || !n_out || (nnzb > 0 && !col_idx) || R <= 0 || C <= 0)
    return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  bsp_spmm_plan p;
  p.M = M;
  p.K = K;
  p.N = N;
  p.R = R;
  p.C = C;
  p.nnzb = nnzb;
  p.strategy = strategy;
  bsp_status s = plan_spmm_host(&p, row_ptr, col_idx, sm_count, max_smem, opts);
  if (s != BSP_OK) return s;
  *n_out = static_cast<int64_t>(p.h_entry_rows.size());
  if (rows_out && !p.h_entry_rows.empty())
    memcpy(rows_out, p.h_entry_rows.data(), p.h_entry_rows.size() * sizeof(int32_t));
  return BSP_OK;
}

bsp_status bsp_sddmm_plan_inspect(int64_t M, int64_t N, int32_t R, int32_t C, int64_t nnzb,
                                  const int32_t* row_ptr, const int32_t* col_idx, int64_t K,
                                  bsp_strategy strategy, const bsp_sddmm_opts* opts,
                                  int32_t sm_count, int32_t max_smem, int64_t info[16],
                                  int32_t* units_out, int32_t* cta_begin_out) {
  if (!row_ptr || !info || (nnzb > 0 && !col_idx) || R <= 0 || C <= 0)
    return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  bsp_sddmm_plan p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.R = R;
  p.C = C;
  p.nnzb = nnzb;
  p.strategy = strategy;
  bsp_status s = plan_sddmm_host(&p, row_ptr, col_idx, sm_count, max_smem, opts);
  if (s != BSP_OK) return s;
  bsp_sddmm_plan_info(&p, info);
  if (units_out) {
    if (p.variant == 1) memcpy(units_out, p.h_rs_units.data(), p.h_rs_units.size() * sizeof(SddmmRsUnit));
    else memcpy(units_out, p.h_units.data(), p.h_units.size() * sizeof(SddmmUnit));
  }
  if (cta_begin_out)
    memcpy(cta_begin_out, p.h_cta_begin.data(), p.h_cta_begin.size() * sizeof(int32_t));
  return BSP_OK;
}

bsp_status bsp_spgemm_plan_inspect(int64_t M, int64_t K, int64_t N, int32_t Ra, int32_t Ca,
                                   int32_t Cb, int64_t a_nnzb, const int32_t* a_row_ptr,
                                   const int32_t* a_col_idx, int64_t b_nnzb,
                                   const int32_t* b_row_ptr, const int32_t* b_col_idx,
                                   const bsp_spmm_opts* opts, int32_t sm_count, int32_t max_smem,
                                   int64_t info[16], int32_t* out_row_ptr, int32_t* out_col_idx,
                                   int32_t* units_out, int32_t* steps_out, int32_t* cta_begin_out) {
  if (!a_row_ptr || !b_row_ptr || !info || (a_nnzb > 0 && !a_col_idx) || (b_nnzb > 0 && !b_col_idx))
    return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  bsp_spgemm_plan p;
  p.M = M;
  p.K = K;
  p.N = N;
  p.Ra = Ra;
  p.Ca = Ca;
  p.Cb = Cb;
  p.nnzb_a = a_nnzb;
  p.nnzb_b = b_nnzb;
  bsp_status s = plan_spgemm_host(&p, a_row_ptr, a_col_idx, b_row_ptr, b_col_idx, sm_count, max_smem, opts);
  if (s != BSP_OK) return s;
  bsp_spgemm_plan_info(&p, info);
  if (out_row_ptr) memcpy(out_row_ptr, p.out_row_ptr.data(), p.out_row_ptr.size() * sizeof(int32_t));
  if (out_col_idx && !p.out_col_idx.empty())
    memcpy(out_col_idx, p.out_col_idx.data(), p.out_col_idx.size() * sizeof(int32_t));
  if (units_out && !p.h_units.empty()) memcpy(units_out, p.h_units.data(), p.h_units.size() * sizeof(SpgemmUnit));
  if (steps_out && !p.h_steps.empty()) memcpy(steps_out, p.h_steps.data(), p.h_steps.size() * sizeof(SpgemmStep));
  if (cta_begin_out) memcpy(cta_begin_out, p.h_cta_begin.data(), p.h_cta_begin.size() * sizeof(int32_t));
  return BSP_OK;
}

bsp_status bsp_attn_plan_inspect(int64_t S, int64_t d, int64_t nnzb, const int32_t* row_ptr,
                                 const int32_t* col_idx, const bsp_spmm_opts* opts, int32_t sm_count,
                                 int32_t max_smem, int64_t info[16], int32_t* units_out,
                                 int32_t* chunks_out, int32_t* cta_begin_out) {
  if (!row_ptr || !info || (nnzb > 0 && !col_idx)) return set_error(BSP_ERR_INVALID_ARG, "bad arguments");
  bsp_attn_plan p;
  p.S = S;
  p.d = d;
  p.nnzb = nnzb;
  bsp_status s = plan_attn_host(&p, row_ptr, col_idx, sm_count, max_smem, opts);
  if (s != BSP_OK) return s;
  bsp_attn_plan_info(&p, info);
  if (units_out && !p.h_units.empty()) memcpy(units_out, p.h_units.data(), p.h_units.size() * sizeof(AttnUnit));
  if (chunks_out && !p.h_chunks.empty())
    memcpy(chunks_out, p.h_chunks.data(), p.h_chunks.size() * sizeof(AttnChunk));
  if (cta_begin_out) memcpy(cta_begin_out, p.h_cta_begin.data(), p.h_cta_begin.size() * sizeof(int32_t));
  return BSP_OK;
}

}  // extern "C"
