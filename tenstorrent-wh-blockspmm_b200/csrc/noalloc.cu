// bsp_spmm_noalloc: SpMM that allocates no device memory.
//
// Callers that cannot call cudaMalloc -- code running under an allocator that
// owns all device memory (a framework's caching allocator or a memory pool
// sized up front), or a process whose memory budget is fixed before it
// starts -- can still run the Naive/SnF SpMM kernel through this entry point.
// They pass inputs and outputs; the kernel's scratch (its work schedule and
// its status word) lives in the fixed-size device array below instead of a
// per-call allocation.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds it (kScratchBytes) until the process exits.  All calls share
// it and it keeps the previous call's contents, so each call rewrites the
// schedule and zeroes the status word before launching, and two calls whose
// work overlaps on the GPU (different streams, or different host threads on
// one device) race on it.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "bsp_internal.h"

namespace bsp {

int spmm_smem_bytes(int stages, int stage_bytes, bool c_f32);

namespace {

constexpr size_t kScratchBytes = size_t(4) << 20;  // 4 MiB: schedule tables + status word
constexpr size_t kStatusBytes = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// Device address of g_noalloc_scratch per device.  In host code the symbol is
// only a host-side stand-in, so the real address is looked up once per device,
// with that device current.
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};
PFN_encodeTiled g_encode = nullptr;

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

bsp_status setup_current_device(int* ordinal, void** scratch) {
  int dev = 0;
  bsp_status s = cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (s != BSP_OK) return s;
  if (dev < 0 || dev >= kMaxDevices) return set_error(BSP_ERR_UNSUPPORTED, "device ordinal too large");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    s = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
    if (s != BSP_OK) return s;
    g_scratch_addr[dev] = p;
  }
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return set_error(BSP_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
    g_encode = reinterpret_cast<PFN_encodeTiled>(fn);
  }
  *ordinal = dev;
  *scratch = g_scratch_addr[dev];
  return BSP_OK;
}

}  // namespace
}  // namespace bsp

using namespace bsp;

extern "C" bsp_status bsp_spmm_noalloc(const bsp_bsr_desc* A, const int32_t* host_row_ptr,
                                       const int32_t* host_col_idx, const void* B, int64_t ldb,
                                       void* C, int64_t ldc, int64_t N, bsp_dtype c_type,
                                       bsp_strategy strategy, void* stream) {
  if (!A || !host_row_ptr || (A->nnzb > 0 && !host_col_idx) || !B || !C)
    return set_error(BSP_ERR_INVALID_ARG, "null argument");
  if (strategy != BSP_NAIVE && strategy != BSP_SNF)
    return set_error(BSP_ERR_UNSUPPORTED, "bsp_spmm_noalloc runs the Naive and SnF strategies");
  if (A->R <= 0 || A->C <= 0 || A->rows <= 0 || A->cols <= 0 || A->nnzb < 0 ||
      (A->nnzb > 0 && !A->values) || A->rows % A->R || A->cols % A->C || !A->row_ptr ||
      (A->nnzb > 0 && !A->col_idx))
    return set_error(BSP_ERR_INVALID_ARG, "bad BSR descriptor");
  if (A->values && reinterpret_cast<uintptr_t>(A->values) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "BSR values must be 16-byte aligned");
  if (c_type != BSP_BF16 && c_type != BSP_F32)
    return set_error(BSP_ERR_INVALID_ARG, "C type must be BSP_BF16 or BSP_F32");
  if (ldb < N || ldc < N) return set_error(BSP_ERR_INVALID_ARG, "leading dimensions must be >= N");
  int ordinal = 0;
  void* scratch = nullptr;
  bsp_status s = setup_current_device(&ordinal, &scratch);
  if (s != BSP_OK) return s;

  int sm_count = 0, max_smem = 0;
  if ((s = cuda_check(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, ordinal),
                      "cudaDeviceGetAttribute")) != BSP_OK)
    return s;
  if ((s = cuda_check(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, ordinal),
                      "cudaDeviceGetAttribute")) != BSP_OK)
    return s;

  uint8_t* base = static_cast<uint8_t*>(scratch);
  unsigned int* d_status = reinterpret_cast<unsigned int*>(base);
  bsp_device dev;  // borrowed view: no allocation, status word in the scratch array
  dev.ordinal = ordinal;
  dev.sm_count = sm_count;
  dev.max_smem_optin = max_smem;
  dev.encode = g_encode;
  dev.d_status = d_status;

  bsp_spmm_plan plan;
  plan.dev = &dev;
  plan.M = A->rows;
  plan.K = A->cols;
  plan.N = N;
  plan.R = A->R;
  plan.C = A->C;
  plan.nnzb = A->nnzb;
  plan.c_type = c_type;
  plan.strategy = strategy;
  s = plan_spmm_host(&plan, host_row_ptr, host_col_idx, sm_count, max_smem, nullptr);
  if (s != BSP_OK) return s;

  const size_t b_units = align256(plan.h_units.size() * sizeof(SpmmUnit));
  const size_t b_cta = align256(plan.h_cta_begin.size() * sizeof(int32_t));
  const size_t b_steps = align256(plan.h_steps.size() * sizeof(int32_t));
  const size_t need = kStatusBytes + b_units + b_cta + b_steps;
  if (need > kScratchBytes)
    return set_error(BSP_ERR_UNSUPPORTED,
                     "bsp_spmm_noalloc: the schedule needs " + std::to_string(need) +
                         " bytes of scratch, more than the fixed " + std::to_string(kScratchBytes) +
                         " (use bsp_spmm_plan_create, which allocates)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  plan.d_units = reinterpret_cast<SpmmUnit*>(base + kStatusBytes);
  plan.d_cta_begin = reinterpret_cast<int32_t*>(base + kStatusBytes + b_units);
  plan.d_steps = reinterpret_cast<int32_t*>(base + kStatusBytes + b_units + b_cta);
  // The array keeps the last call's contents: rewrite the whole schedule and
  // clear the status word the kernel latches errors into.
  if ((s = cuda_check(cudaMemsetAsync(d_status, 0, kStatusBytes, st), "clear status")) != BSP_OK) return s;
  if ((s = cuda_check(cudaMemcpyAsync(plan.d_units, plan.h_units.data(), plan.h_units.size() * sizeof(SpmmUnit),
                                      cudaMemcpyHostToDevice, st), "upload units")) != BSP_OK)
    return s;
  if ((s = cuda_check(cudaMemcpyAsync(plan.d_cta_begin, plan.h_cta_begin.data(),
                                      plan.h_cta_begin.size() * sizeof(int32_t), cudaMemcpyHostToDevice, st),
                      "upload cta offsets")) != BSP_OK)
    return s;
  if ((s = cuda_check(cudaMemcpyAsync(plan.d_steps, plan.h_steps.data(), plan.h_steps.size() * sizeof(int32_t),
                                      cudaMemcpyHostToDevice, st), "upload steps")) != BSP_OK)
    return s;
  s = launch_spmm(&plan, A, B, ldb, C, ldc, st);
  if (s != BSP_OK) return s;
  // The host schedule buffers must outlive the copies: wait for the stream.
  if ((s = cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize")) != BSP_OK) return s;
  unsigned int bits = 0;
  if ((s = cuda_check(cudaMemcpy(&bits, d_status, sizeof(bits), cudaMemcpyDeviceToHost), "read status")) != BSP_OK)
    return s;
  if (bits) return set_error(BSP_ERR_TIMEOUT, "a kernel wait timed out (status bits " + std::to_string(bits) + ")");
  return BSP_OK;
}
