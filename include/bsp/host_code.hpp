// bsp/host_code.hpp -- the reference's host-code API, implemented over libbsp.
//
// Same names, template parameters, argument lists and registries as the
// reference's block_spmm/inc/host_code.hpp:36-222 (SpMM) and
// block_sddmm/inc/host_code.hpp:43-153 (SDDMM), so that a caller written
// against the Tenstorrent host code compiles against this header.  Differences
// a caller sees:
//   * IDevice is bsp::IDevice (a B200 opened with bsp::CreateDevice).
//   * Inputs are NOT tilized: blocks and dense matrices stay row-major
//     (the reference's tests call tilize_nfaces first, test_block_spmm.cpp:77-78).
//   * Every element of the SpMM output is written, rows of empty block-rows
//     included (the reference relies on the caller zero-filling `output`).
//   * Errors throw std::runtime_error (the reference uses TT_THROW / asserts).
//   * NoC-specific template flags (use_optimal_noc, in0_left_to_right,
//     in1_bottom_to_top) are accepted and have no effect; `verbose` prints the
//     plan, `is_profiling` times 10 kernel runs after a warm-up and prints
//     "Device TFLOP/s: <x>" (as the reference's profiling flow reports).
//   * The ablation variants (*_no_a_read, *_no_b_read, *_no_compute,
//     *_no_write) are not provided: they are Tensix profiling aids.
#pragma once

#include <cstdint>
#include <cstdio>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "bsp.h"
#include "bsp/bsr_matrix.hpp"

namespace bsp {

class IDevice {
 public:
  explicit IDevice(int ordinal) {
    if (bsp_device_open(ordinal, &dev_) != BSP_OK)
      throw std::runtime_error(std::string("bsp: cannot open device: ") + bsp_last_error_string());
  }
  ~IDevice() { bsp_device_close(dev_); }
  IDevice(const IDevice&) = delete;
  IDevice& operator=(const IDevice&) = delete;
  bsp_device* handle() const { return dev_; }

 private:
  bsp_device* dev_ = nullptr;
};

inline IDevice* CreateDevice(int ordinal) { return new IDevice(ordinal); }
inline bool CloseDevice(IDevice* d) {
  delete d;
  return true;
}

inline void check(bsp_status s, const char* what) {
  if (s != BSP_OK)
    throw std::runtime_error(std::string(what) + ": " + bsp_status_string(s) + ": " +
                             bsp_last_error_string());
}

// ---- device buffers (the reference's sparse_common::MakeBuffer) ------------
// A device allocation of `size` bytes on one device, freed when the last
// shared_ptr to it goes: the role of the tt-metal Buffer that the reference's
// MakeBuffer returns (sparse_common/host_code_utils.cpp:5-18).  page_size is
// kept for callers that read it back; device memory is not paged here.
class Buffer {
 public:
  Buffer(IDevice* device, uint64_t size, uint64_t page_size) : dev_(device), size_(size), page_(page_size) {
    check(bsp_buffer_alloc(dev_->handle(), static_cast<int64_t>(size), &ptr_), "MakeBuffer");
  }
  ~Buffer() { bsp_buffer_free(dev_->handle(), ptr_); }
  Buffer(const Buffer&) = delete;
  Buffer& operator=(const Buffer&) = delete;
  void* address() const { return ptr_; }
  uint64_t size() const { return size_; }
  uint64_t page_size() const { return page_; }
  IDevice* device() const { return dev_; }

 private:
  IDevice* dev_;
  void* ptr_ = nullptr;
  uint64_t size_, page_;
};

// Host <-> device copies of a whole buffer (the reference's EnqueueWriteBuffer
// / EnqueueReadBuffer, load_balanced_new_DM.cpp:499-505).  Both complete before
// they return, whatever `blocking` says.
template <typename T>
void EnqueueWriteBuffer(Buffer& buf, const std::vector<T>& src, bool /*blocking*/ = true) {
  if (src.size() * sizeof(T) > buf.size()) throw std::runtime_error("bsp: EnqueueWriteBuffer: source larger than buffer");
  check(bsp_buffer_write(buf.device()->handle(), buf.address(), src.data(),
                         static_cast<int64_t>(src.size() * sizeof(T))),
        "EnqueueWriteBuffer");
}
template <typename T>
void EnqueueReadBuffer(Buffer& buf, std::vector<T>& dst, bool /*blocking*/ = true) {
  dst.resize(buf.size() / sizeof(T));
  check(bsp_buffer_read(buf.device()->handle(), dst.data(), buf.address(),
                        static_cast<int64_t>(dst.size() * sizeof(T))),
        "EnqueueReadBuffer");
}

// A BSR matrix resident on the device (bsp_bsr_upload / bsp_bsr_free): upload
// once, then run any number of plans on desc().
class DeviceBsr {
 public:
  DeviceBsr(IDevice* device, const bsr_matrix<bfloat16>& a, bool with_values = true) : dev_(device) {
    std::vector<uint16_t> v;
    if (with_values) {
      v.resize(a.data.size());
      for (size_t i = 0; i < v.size(); ++i) v[i] = a.data[i].to_uint16();
    }
    check(bsp_bsr_upload(dev_->handle(), static_cast<int64_t>(a.H), static_cast<int64_t>(a.W),
                         static_cast<int32_t>(a.R), static_cast<int32_t>(a.C), static_cast<int64_t>(a.nblocks),
                         a.indptr.data(), a.indices.data(), with_values ? v.data() : nullptr, &desc_),
          "bsp_bsr_upload");
  }
  ~DeviceBsr() { bsp_bsr_free(dev_->handle(), &desc_); }
  DeviceBsr(const DeviceBsr&) = delete;
  DeviceBsr& operator=(const DeviceBsr&) = delete;
  const bsp_bsr_desc& desc() const { return desc_; }

 private:
  IDevice* dev_;
  bsp_bsr_desc desc_{};
};

namespace detail {

inline std::vector<uint16_t> bits(const std::vector<bfloat16>& v) {
  std::vector<uint16_t> out(v.size());
  for (size_t i = 0; i < v.size(); ++i) out[i] = v[i].to_uint16();
  return out;
}

template <bool verbose, bool is_profiling>
void spmm(bsr_matrix<bfloat16>& a, dense_matrix<bfloat16>& b, dense_matrix<bfloat16>& output,
          bool bcast_batch, uint32_t nnz_blocks, uint32_t M, uint32_t N, uint32_t K, uint32_t R,
          uint32_t C, uint32_t B, IDevice* device, bsp_strategy strategy, int no_lb,
          const char* name) {
  if (bcast_batch || B != 1) throw std::runtime_error("bsp: batched SpMM (B != 1) is not supported");
  if (a.H != M || a.W != K || a.R != R || a.C != C || b.H != K || b.W != N || a.nblocks != nnz_blocks)
    throw std::runtime_error("bsp: SpMM arguments do not match the operands");
  if (output.H != M || output.W != N) output = dense_matrix<bfloat16>(static_cast<int>(M), static_cast<int>(N));
  const std::vector<uint16_t> av = bits(a.data), bv = bits(b.data);
  std::vector<uint16_t> cv(static_cast<size_t>(M) * N);
  bsp_spmm_opts opts{};
  opts.no_load_balance = no_lb;
  if (verbose) std::printf("[bsp] %s: M=%u N=%u K=%u R=%u C=%u nnz_blocks=%u\n", name, M, N, K, R, C, nnz_blocks);
  if (is_profiling) {
    double ms = 0;
    check(bsp_spmm_host_profile(device->handle(), M, K, static_cast<int32_t>(R), static_cast<int32_t>(C),
                                static_cast<int64_t>(a.nblocks), a.indptr.data(), a.indices.data(),
                                av.data(), bv.data(), N, cv.data(), strategy, &opts, 10, &ms),
          name);
    const double tflops = 2.0 * a.nblocks * R * C * N / (ms * 1e-3) / 1e12;
    std::printf("Device TFLOP/s: %.3f\n", tflops);
  } else {
    check(bsp_spmm_host(device->handle(), M, K, static_cast<int32_t>(R), static_cast<int32_t>(C),
                        static_cast<int64_t>(a.nblocks), a.indptr.data(), a.indices.data(), av.data(),
                        bv.data(), N, cv.data(), strategy, &opts),
          name);
  }
  for (size_t i = 0; i < cv.size(); ++i) output.data[i] = bfloat16::from_bits(cv[i]);
}

template <bool verbose, bool is_profiling>
void sddmm(bsr_matrix<bfloat16>& mask, dense_matrix<bfloat16>& c, dense_matrix<bfloat16>& d,
           bsr_matrix<bfloat16>& output, uint32_t M, uint32_t N, uint32_t K, uint32_t R,
           uint32_t C_block, uint32_t B, IDevice* device, bsp_strategy strategy, const char* name) {
  if (B != 1) throw std::runtime_error("bsp: batched SDDMM (B != 1) is not supported");
  if (mask.H != M || mask.W != N || mask.R != R || mask.C != C_block || c.H != M || c.W != K ||
      d.H != K || d.W != N)
    throw std::runtime_error("bsp: SDDMM arguments do not match the operands");
  const std::vector<uint16_t> mv = bits(mask.data), cv = bits(c.data), dv = bits(d.data);
  std::vector<uint16_t> out(mask.nblocks * R * C_block);
  if (verbose) std::printf("[bsp] %s: M=%u N=%u K=%u R=%u C=%u nnz_blocks=%zu\n", name, M, N, K, R, C_block, mask.nblocks);
  if (is_profiling) {
    double ms = 0;
    check(bsp_sddmm_host_profile(device->handle(), M, N, static_cast<int32_t>(R), static_cast<int32_t>(C_block),
                                 static_cast<int64_t>(mask.nblocks), mask.indptr.data(), mask.indices.data(),
                                 mv.empty() ? nullptr : mv.data(), cv.data(), dv.data(), K, out.data(),
                                 strategy, nullptr, 10, &ms),
          name);
    const double tflops = (2.0 * mask.nblocks * R * C_block * K + 1.0 * mask.nblocks * R * C_block) / (ms * 1e-3) / 1e12;
    std::printf("Device TFLOP/s: %.3f\n", tflops);
  } else {
    check(bsp_sddmm_host(device->handle(), M, N, static_cast<int32_t>(R), static_cast<int32_t>(C_block),
                         static_cast<int64_t>(mask.nblocks), mask.indptr.data(), mask.indices.data(),
                         mv.empty() ? nullptr : mv.data(), cv.data(), dv.data(), K, out.data(), strategy, nullptr),
          name);
  }
  std::vector<bfloat16> vals(out.size());
  for (size_t i = 0; i < out.size(); ++i) vals[i] = bfloat16::from_bits(out[i]);
  output = bsr_matrix<bfloat16>(std::move(vals), mask.indptr, mask.indices, M, N, R, C_block, mask.nblocks);
}

}  // namespace detail

// C = a * b for two BSR matrices on the GPU: the device form of the
// reference's bsr_matrix<T>::spgemm (sparse_common/bsr_matrix.hpp:741-810),
// same result pattern (columns ascending per block-row) and one bf16 rounding
// per block.  Block sizes 32, 64 or 128; a.W == b.H and a.C == b.R.
inline bsr_matrix<bfloat16> spgemm(bsr_matrix<bfloat16>& a, bsr_matrix<bfloat16>& b, IDevice* device,
                                   const bsp_spmm_opts* opts = nullptr) {
  if (a.W != b.H || a.C != b.R) throw std::runtime_error("bsp: spgemm operands do not chain");
  const std::vector<uint16_t> av = detail::bits(a.data), bv = detail::bits(b.data);
  int64_t nnzb = 0;
  check(bsp_spgemm_host(device->handle(), a.H, a.W, b.W, static_cast<int32_t>(a.R), static_cast<int32_t>(a.C),
                        static_cast<int32_t>(b.C), static_cast<int64_t>(a.nblocks), a.indptr.data(),
                        a.indices.data(), av.data(), static_cast<int64_t>(b.nblocks), b.indptr.data(),
                        b.indices.data(), bv.data(), 0, &nnzb, nullptr, nullptr, nullptr, opts, 0, nullptr),
        "bsp_spgemm_host (size)");
  std::vector<int> rp(a.H / a.R + 1), ci(static_cast<size_t>(nnzb));
  std::vector<uint16_t> out(static_cast<size_t>(nnzb) * a.R * b.C);
  check(bsp_spgemm_host(device->handle(), a.H, a.W, b.W, static_cast<int32_t>(a.R), static_cast<int32_t>(a.C),
                        static_cast<int32_t>(b.C), static_cast<int64_t>(a.nblocks), a.indptr.data(),
                        a.indices.data(), av.data(), static_cast<int64_t>(b.nblocks), b.indptr.data(),
                        b.indices.data(), bv.data(), nnzb, &nnzb, rp.data(), ci.data(), out.data(), opts, 0,
                        nullptr),
        "bsp_spgemm_host");
  std::vector<bfloat16> vals(out.size());
  for (size_t i = 0; i < out.size(); ++i) vals[i] = bfloat16::from_bits(out[i]);
  return bsr_matrix<bfloat16>(std::move(vals), std::move(rp), std::move(ci), a.H, b.W, a.R, b.C,
                              static_cast<size_t>(nnzb));
}

// O = softmax_rows(scale * Q K^T on the mask's blocks) V, one head: the
// reference's SDDMM -> row softmax -> SpMM chain fused on the GPU.  mask: S x S
// with 32 x 32 blocks (values ignored); Q, K, V: S x d (d = 64 or 128).
inline dense_matrix<bfloat16> attention_step(bsr_matrix<bfloat16>& mask, dense_matrix<bfloat16>& q,
                                             dense_matrix<bfloat16>& k, dense_matrix<bfloat16>& v, float scale,
                                             IDevice* device) {
  if (mask.H != mask.W || mask.R != 32 || mask.C != 32 || q.H != mask.H || k.H != q.H || v.H != q.H ||
      k.W != q.W || v.W != q.W)
    throw std::runtime_error("bsp: attention_step operands do not match");
  const std::vector<uint16_t> qv = detail::bits(q.data), kv = detail::bits(k.data), vv = detail::bits(v.data);
  std::vector<uint16_t> o(qv.size());
  check(bsp_attn_host(device->handle(), static_cast<int64_t>(mask.H), static_cast<int64_t>(q.W),
                      static_cast<int64_t>(mask.nblocks),
                      mask.indptr.data(), mask.indices.data(), qv.data(), kv.data(), vv.data(), scale, o.data(),
                      nullptr),
        "bsp_attn_host");
  dense_matrix<bfloat16> out(static_cast<int>(q.H), static_cast<int>(q.W));
  for (size_t i = 0; i < o.size(); ++i) out.data[i] = bfloat16::from_bits(o[i]);
  return out;
}

}  // namespace bsp

namespace sparse_common {

// sparse_common/host_code_utils.cpp:5-11: `size` bytes with pages of
// `page_size` bytes.  `sram` asked tt-metal for core-local L1; a B200 has no
// addressable equivalent for a buffer (its 126 MB L2 caches device memory by
// itself), so the buffer is device memory either way.
inline std::shared_ptr<bsp::Buffer> MakeBuffer(bsp::IDevice* device, uint32_t size, uint32_t page_size,
                                               bool /*sram*/ = false) {
  return std::make_shared<bsp::Buffer>(device, size, page_size);
}

// sparse_common/host_code_utils.cpp:13-18: n_tiles 32 x 32 tiles of
// element_size-byte elements.
inline std::shared_ptr<bsp::Buffer> MakeBuffer(bsp::IDevice* device, uint32_t n_tiles, size_t element_size,
                                               bool sram = false) {
  const uint32_t tile = static_cast<uint32_t>(element_size) * 32u * 32u;
  return MakeBuffer(device, tile * n_tiles, sram ? tile * n_tiles : tile, sram);
}

}  // namespace sparse_common

namespace bsr_host_code {

using bsp::IDevice;
using sparse_common::MakeBuffer;

// Paper name "Naive" (block_spmm/inc/host_code.hpp:36-50).
template <bool verbose = false, bool is_profiling = false, bool use_optimal_noc = true>
void bsr_spmm_multicore_load_balanced_new_DM(bsr_matrix<bfloat16>& a, dense_matrix<bfloat16>& b,
                                             dense_matrix<bfloat16>& output, bool bcast_batch,
                                             uint32_t nnz_blocks, uint32_t M, uint32_t N, uint32_t K,
                                             uint32_t R, uint32_t C, uint32_t B, IDevice* device) {
  bsp::detail::spmm<verbose, is_profiling>(a, b, output, bcast_batch, nnz_blocks, M, N, K, R, C, B, device,
                                           BSP_NAIVE, 0, "bsr_spmm_multicore_load_balanced_new_DM");
}

// Paper name "SnF in0 naive in1" (host_code.hpp:52-66).
template <bool verbose = false, bool is_profiling = false, bool use_optimal_noc = true>
void bsr_spmm_multicore_snf(bsr_matrix<bfloat16>& a, dense_matrix<bfloat16>& b,
                            dense_matrix<bfloat16>& output, bool bcast_batch, uint32_t nnz_blocks,
                            uint32_t M, uint32_t N, uint32_t K, uint32_t R, uint32_t C, uint32_t B,
                            IDevice* device) {
  bsp::detail::spmm<verbose, is_profiling>(a, b, output, bcast_batch, nnz_blocks, M, N, K, R, C, B, device,
                                           BSP_SNF, 0, "bsr_spmm_multicore_snf");
}

// Paper name "SnF in0 CDA in1" = "DDA" (host_code.hpp:68-83).
template <bool verbose = false, bool is_profiling = false, bool use_optimal_noc = true,
          bool in0_left_to_right = true, bool in1_bottom_to_top = true>
void bsr_spmm_multicore_snfin0_cdain1(bsr_matrix<bfloat16>& a, dense_matrix<bfloat16>& b,
                                      dense_matrix<bfloat16>& output, bool bcast_batch,
                                      uint32_t nnz_blocks, uint32_t M, uint32_t N, uint32_t K,
                                      uint32_t R, uint32_t C, uint32_t B, IDevice* device) {
  bsp::detail::spmm<verbose, is_profiling>(a, b, output, bcast_batch, nnz_blocks, M, N, K, R, C, B, device,
                                           BSP_DDA, 0, "bsr_spmm_multicore_snfin0_cdain1");
}

// No-load-balance variants (host_code.hpp:113-161): contiguous work split.
template <bool verbose = false, bool is_profiling = false, bool use_optimal_noc = true>
void bsr_spmm_multicore_load_balanced_new_DM_no_lb(bsr_matrix<bfloat16>& a, dense_matrix<bfloat16>& b,
                                                   dense_matrix<bfloat16>& output, bool bcast_batch,
                                                   uint32_t nnz_blocks, uint32_t M, uint32_t N,
                                                   uint32_t K, uint32_t R, uint32_t C, uint32_t B,
                                                   IDevice* device) {
  bsp::detail::spmm<verbose, is_profiling>(a, b, output, bcast_batch, nnz_blocks, M, N, K, R, C, B, device,
                                           BSP_NAIVE, 1, "bsr_spmm_multicore_load_balanced_new_DM_no_lb");
}

template <bool verbose = false, bool is_profiling = false, bool use_optimal_noc = true>
void bsr_spmm_multicore_snf_no_lb(bsr_matrix<bfloat16>& a, dense_matrix<bfloat16>& b,
                                  dense_matrix<bfloat16>& output, bool bcast_batch, uint32_t nnz_blocks,
                                  uint32_t M, uint32_t N, uint32_t K, uint32_t R, uint32_t C, uint32_t B,
                                  IDevice* device) {
  bsp::detail::spmm<verbose, is_profiling>(a, b, output, bcast_batch, nnz_blocks, M, N, K, R, C, B, device,
                                           BSP_SNF, 1, "bsr_spmm_multicore_snf_no_lb");
}

template <bool verbose = false, bool is_profiling = false, bool use_optimal_noc = true,
          bool in0_left_to_right = true, bool in1_bottom_to_top = true>
void bsr_spmm_multicore_snfin0_cdain1_no_lb(bsr_matrix<bfloat16>& a, dense_matrix<bfloat16>& b,
                                            dense_matrix<bfloat16>& output, bool bcast_batch,
                                            uint32_t nnz_blocks, uint32_t M, uint32_t N, uint32_t K,
                                            uint32_t R, uint32_t C, uint32_t B, IDevice* device) {
  bsp::detail::spmm<verbose, is_profiling>(a, b, output, bcast_batch, nnz_blocks, M, N, K, R, C, B, device,
                                           BSP_DDA, 1, "bsr_spmm_multicore_snfin0_cdain1_no_lb");
}

// block_spmm/inc/host_code.hpp:165-177
using HostCodeFunctionPtr = void (*)(bsr_matrix<bfloat16>& a, dense_matrix<bfloat16>& b,
                                     dense_matrix<bfloat16>& output, bool bcast_batch,
                                     uint32_t nnz_blocks, uint32_t M, uint32_t N, uint32_t K,
                                     uint32_t R, uint32_t C, uint32_t B, IDevice* device);

// Indices as in the reference (host_code.hpp:182-190): 0=Naive, 1=SnF, 2=CDA,
// 3=CDA no_lb, 4=Naive no_lb, 5=SnF no_lb.
static std::pair<HostCodeFunctionPtr, std::string> HostCodeRegistryVerbose[] = {
    {bsr_spmm_multicore_load_balanced_new_DM<true, false>, "bsr_spmm_multicore_load_balanced_new_DM"},
    {bsr_spmm_multicore_snf<true, false>, "bsr_spmm_multicore_snf"},
    {bsr_spmm_multicore_snfin0_cdain1<true, false>, "bsr_spmm_multicore_snfin0_cdain1"},
    {bsr_spmm_multicore_snfin0_cdain1_no_lb<true, false>, "bsr_spmm_multicore_snfin0_cdain1_no_lb"},
    {bsr_spmm_multicore_load_balanced_new_DM_no_lb<true, false>, "bsr_spmm_multicore_load_balanced_new_DM_no_lb"},
    {bsr_spmm_multicore_snf_no_lb<true, false>, "bsr_spmm_multicore_snf_no_lb"},
};

// The full algorithms and their no-load-balance variants of the reference's
// profiling registry (host_code.hpp:195-221, entries 0-2 and 15-17); the
// Tensix ablation entries 3-14 have no B200 counterpart.
static std::pair<HostCodeFunctionPtr, std::string> HostCodeRegistryProfiling[] = {
    {bsr_spmm_multicore_load_balanced_new_DM<false, true>, "bsr_spmm_multicore_load_balanced_new_DM"},
    {bsr_spmm_multicore_snf<false, true>, "bsr_spmm_multicore_snf"},
    {bsr_spmm_multicore_snfin0_cdain1<false, true>, "bsr_spmm_multicore_snfin0_cdain1"},
    {bsr_spmm_multicore_snfin0_cdain1_no_lb<false, true>, "bsr_spmm_multicore_snfin0_cdain1_no_lb"},
    {bsr_spmm_multicore_load_balanced_new_DM_no_lb<false, true>, "bsr_spmm_multicore_load_balanced_new_DM_no_lb"},
    {bsr_spmm_multicore_snf_no_lb<false, true>, "bsr_spmm_multicore_snf_no_lb"},
};

}  // namespace bsr_host_code

namespace bsr_sddmm_host_code {

using bsp::IDevice;

// block_sddmm/inc/host_code.hpp:43-56
template <bool verbose = false, bool is_profiling = false>
void bsr_sddmm_multicore_naive(bsr_matrix<bfloat16>& sampling_mask, dense_matrix<bfloat16>& c,
                               dense_matrix<bfloat16>& d, bsr_matrix<bfloat16>& output, uint32_t M,
                               uint32_t N, uint32_t K, uint32_t R, uint32_t C_block, uint32_t B,
                               IDevice* device) {
  bsp::detail::sddmm<verbose, is_profiling>(sampling_mask, c, d, output, M, N, K, R, C_block, B, device,
                                            BSP_NAIVE, "bsr_sddmm_multicore_naive");
}

// block_sddmm/inc/host_code.hpp:58-71
template <bool verbose = false, bool is_profiling = false>
void bsr_sddmm_multicore_CDA(bsr_matrix<bfloat16>& sampling_mask, dense_matrix<bfloat16>& c,
                             dense_matrix<bfloat16>& d, bsr_matrix<bfloat16>& output, uint32_t M,
                             uint32_t N, uint32_t K, uint32_t R, uint32_t C_block, uint32_t B,
                             IDevice* device) {
  bsp::detail::sddmm<verbose, is_profiling>(sampling_mask, c, d, output, M, N, K, R, C_block, B, device,
                                            BSP_DDA, "bsr_sddmm_multicore_CDA");
}

// block_sddmm/inc/host_code/bsr_sddmm_multicore_SnF_C.cpp: the reference's
// unfinished store-and-forward SDDMM (excluded from its build by
// block_sddmm/inc/host_code/CMakeLists.txt:7, not in its registries).  Here it
// runs: each CTA keeps a row group's 128 x K panel of c resident while the
// group's d segments stream past, over contiguous runs of units balanced by
// weight.  Not added to the registries below, so their indices stay the
// reference's.
template <bool verbose = false, bool is_profiling = false>
void bsr_sddmm_multicore_SnF(bsr_matrix<bfloat16>& sampling_mask, dense_matrix<bfloat16>& c,
                             dense_matrix<bfloat16>& d, bsr_matrix<bfloat16>& output, uint32_t M,
                             uint32_t N, uint32_t K, uint32_t R, uint32_t C_block, uint32_t B,
                             IDevice* device) {
  bsp::detail::sddmm<verbose, is_profiling>(sampling_mask, c, d, output, M, N, K, R, C_block, B, device,
                                            BSP_SNF, "bsr_sddmm_multicore_SnF");
}

// block_sddmm/inc/host_code.hpp:104-115
using SDDMMHostCodeFunctionPtr = void (*)(bsr_matrix<bfloat16>& sampling_mask, dense_matrix<bfloat16>& c,
                                          dense_matrix<bfloat16>& d, bsr_matrix<bfloat16>& output,
                                          uint32_t M, uint32_t N, uint32_t K, uint32_t R,
                                          uint32_t C_block, uint32_t B, IDevice* device);

// block_sddmm/inc/host_code.hpp:117-125
static std::pair<SDDMMHostCodeFunctionPtr, std::string> HostCodeRegistry[] = {
    {bsr_sddmm_multicore_naive<false, false>, "bsr_sddmm_multicore_naive"},
    {bsr_sddmm_multicore_CDA<false, false>, "bsr_sddmm_multicore_CDA"},
};

static std::pair<SDDMMHostCodeFunctionPtr, std::string> HostCodeRegistryVerbose[] = {
    {bsr_sddmm_multicore_naive<true, false>, "bsr_sddmm_multicore_naive"},
    {bsr_sddmm_multicore_CDA<true, false>, "bsr_sddmm_multicore_CDA"},
};

// Full algorithms of block_sddmm/inc/host_code.hpp:133-153 (entries 0-1).
static std::pair<SDDMMHostCodeFunctionPtr, std::string> HostCodeRegistryProfiling[] = {
    {bsr_sddmm_multicore_naive<false, true>, "bsr_sddmm_multicore_naive"},
    {bsr_sddmm_multicore_CDA<false, true>, "bsr_sddmm_multicore_CDA"},
};

}  // namespace bsr_sddmm_host_code
