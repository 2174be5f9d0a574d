// BSR SDDMM on sm_100a tensor cores:
//   out(i, j) = mask(i, j) (.) (A[iR:(i+1)R, :] * B[:, jC:(j+1)C])   for every mask block (i, j).
//
// Reference path replaced: block_sddmm/inc/host_code/bsr_sddmm_multicore_{naive,CDA}.cpp
// and their Tensix kernels; device hot loop block_sddmm/kernels/compute/
// sddmm_block_multiply.cpp:72-193 (matmul over K steps, Hadamard with the mask).
//
// Mapping ("swap AB"): the 128-row MMA dimension is filled with FOUR output
// segments, each 32 consecutive output columns of one mask block of block-row
// i (segments of different blocks, or of one wide block).  Operand A of the
// MMA is those four B column segments (K x 32 each, MN-major, 64B swizzle),
// operand B is the A row slab A[iR + r_off : +Rs, k-chunk] (K-major), and
// the fp32 accumulator in TMEM holds 128 lanes (= 4 x 32 output columns) x Rs
// rows.  The epilogue multiplies by the mask value in fp32, rounds once to
// bf16 and writes the blocks in mask order (the output keeps the mask pattern).
//
// Warp roles as in spmm.cu: warp 0 TMA, warp 1 MMA, warps 2..5 epilogue
// (epilogue warp with TMEM quarter q owns segment q).
#include <cuda_bf16.h>

#include "bsp_internal.h"
#include "bsp_ptx.cuh"

namespace bsp {
using namespace dev;

namespace {

constexpr int kThreads = 192;
constexpr int kMaxStages = 32;

struct SddmmSmemHeader {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(SddmmSmemHeader) <= 1024, "header must fit its 1 KiB slot");

__device__ __forceinline__ uint32_t bar_addr(const uint64_t* b) { return smem_u32(b); }

__device__ __noinline__ bool drain_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl) {
  int zero = 0;
  WaitCtl c2{&zero, ctl.status, ctl.timeout_ns};
  return mbar_wait_bounded(bar, parity, c2, ST_TIMEOUT_DRAIN);
}

__device__ __forceinline__ void sddmm_producer(const SddmmKernelParams& p, SddmmSmemHeader* hdr,
                                               uint32_t stage0, int u_begin, int u_end,
                                               const WaitCtl& ctl) {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t armed = 0, armed_parity = 0;
  const uint32_t seg_bytes = static_cast<uint32_t>(p.kc * 64);
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    const SddmmUnit un = p.units[u];
#pragma unroll 1
    for (int kci = 0; kci < p.nkc; ++kci) {
      if (!mbar_wait_bounded(bar_addr(&hdr->empty[stage]), phase ^ 1u, ctl, ST_TIMEOUT_PRODUCER))
        goto drain;
      {
        const uint32_t sb = stage0 + static_cast<uint32_t>(stage) * p.stage_bytes;
        const uint32_t full = bar_addr(&hdr->full[stage]);
        mbar_arrive_expect_tx(full, static_cast<uint32_t>(p.a_bytes) + un.nseg * seg_bytes);
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        tma_load_2d(sb, &p.tm_a, kci * p.kc, un.row * p.R + un.r_off, full);
#pragma unroll 1
        for (int q = 0; q < un.nseg; ++q)
          tma_load_2d(sb + p.a_bytes + q * seg_bytes, &p.tm_b, un.col[q], kci * p.kc, full);
      }
      if (++stage == p.stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
drain:
#pragma unroll 1
  for (int s = 0; s < p.stages; ++s)
    if (armed & (1u << s)) drain_wait(bar_addr(&hdr->full[s]), (armed_parity >> s) & 1u, ctl);
}

__device__ __forceinline__ void sddmm_mma(const SddmmKernelParams& p, SddmmSmemHeader* hdr,
                                          uint32_t stage0, uint32_t tmem_base, int u_begin,
                                          int u_end, const WaitCtl& ctl) {
  int stage = 0;
  uint32_t phase = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  const uint32_t idesc = idesc_bf16_f32(128, p.Rs, /*a MN-major*/ 1, /*b K-major*/ 0);
  const uint32_t seg_bytes = static_cast<uint32_t>(p.kc * 64);
  const uint32_t a_sbo = (p.a_swizzle_mode == 2) ? 1024u : 512u;
  const int ksteps = p.kc / 16;
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    if (!mbar_wait_bounded(bar_addr(&hdr->acc_empty[acc]), acc_phase ^ 1u, ctl, ST_TIMEOUT_MMA))
      goto out;
    tc_fence_after();
    {
      const uint32_t d = tmem_base + static_cast<uint32_t>(acc * p.Rs);
#pragma unroll 1
      for (int kci = 0; kci < p.nkc; ++kci) {
        if (!mbar_wait_bounded(bar_addr(&hdr->full[stage]), phase, ctl, ST_TIMEOUT_MMA)) goto out;
        tc_fence_after();
        const uint32_t sb = stage0 + static_cast<uint32_t>(stage) * p.stage_bytes;
#pragma unroll 1
        for (int k = 0; k < ksteps; ++k) {
          // Four 32-column segments, MN-major 64B swizzle: LBO = one segment,
          // SBO = 8 k-rows of 64 B; 16 k-rows per MMA.
          const uint64_t adesc = smem_desc(sb + p.a_bytes + k * 1024u, seg_bytes, 512u, 4u);
          const uint64_t bdesc =
              smem_desc(sb + k * 32u, 16u, a_sbo, static_cast<uint32_t>(p.a_swizzle_mode));
          mma_bf16(d, adesc, bdesc, idesc, (kci | k) != 0);
        }
        mma_commit(bar_addr(&hdr->empty[stage]));
        if (++stage == p.stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    mma_commit(bar_addr(&hdr->acc_full[acc]));
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1u;
  }
out:
  mma_commit(bar_addr(&hdr->drain));
  drain_wait(bar_addr(&hdr->drain), 0, ctl);
}

__device__ __forceinline__ void sddmm_epilogue(const SddmmKernelParams& p, SddmmSmemHeader* hdr,
                                               uint32_t tmem_base, int u_begin, int u_end,
                                               const WaitCtl& ctl, int warp, int lane) {
  const int q = warp & 3;
  int acc = 0;
  uint32_t acc_phase = 0;
  const int64_t blk_elems = static_cast<int64_t>(p.R) * p.C;
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    const SddmmUnit un = p.units[u];
    if (!mbar_wait_bounded(bar_addr(&hdr->acc_full[acc]), acc_phase, ctl, ST_TIMEOUT_EPILOGUE))
      break;
    tc_fence_after();
    if (q < un.nseg) {
      const int64_t blk = un.blk[q];
      const int c = un.col[q] % p.C + lane;  // column inside the block
#pragma unroll 1
      for (int rc = 0; rc < p.Rs / 32; ++rc) {
        uint32_t v[32];
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                               static_cast<uint32_t>(acc * p.Rs + rc * 32);
        tmem_ld_32x32b_x32(taddr, v);
        tmem_ld_wait();
        const int64_t e0 = blk * blk_elems + static_cast<int64_t>(un.r_off + rc * 32) * p.C + c;
        if (p.mask_vals) {
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const int64_t e = e0 + static_cast<int64_t>(r) * p.C;
            const float m = __uint_as_float(static_cast<uint32_t>(p.mask_vals[e]) << 16);
            p.out_vals[e] = __bfloat16_as_ushort(__float2bfloat16_rn(m * __uint_as_float(v[r])));
          }
        } else {
#pragma unroll
          for (int r = 0; r < 32; ++r)
            p.out_vals[e0 + static_cast<int64_t>(r) * p.C] =
                __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[r])));
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_addr(&hdr->acc_empty[acc]));
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1u;
  }
}

__global__ void __launch_bounds__(kThreads, 1) sddmm_bsr_tcgen05(const __grid_constant__ SddmmKernelParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  SddmmSmemHeader* hdr = reinterpret_cast<SddmmSmemHeader*>(gbase);
  const uint32_t stage0 = base + 1024u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int u_begin = p.cta_begin[blockIdx.x];
  const int u_end = p.cta_begin[blockIdx.x + 1];

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(bar_addr(&hdr->full[s]), 1);
      mbar_init(bar_addr(&hdr->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_addr(&hdr->acc_full[a]), 1);
      mbar_init(bar_addr(&hdr->acc_empty[a]), 4);
    }
    mbar_init(bar_addr(&hdr->drain), 1);
    hdr->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&hdr->tmem_base), static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = hdr->tmem_base;
  const WaitCtl ctl{&hdr->abort_flag, p.status, p.timeout_ns};

  if (warp == 0) {
    if (lane == 0) sddmm_producer(p, hdr, stage0, u_begin, u_end, ctl);
  } else if (warp == 1) {
    if (lane == 0) sddmm_mma(p, hdr, stage0, tmem_base, u_begin, u_end, ctl);
  } else {
    sddmm_epilogue(p, hdr, tmem_base, u_begin, u_end, ctl, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
}

}  // namespace

int sddmm_smem_bytes(int stages, int stage_bytes) { return 1024 + 1024 + stages * stage_bytes; }

bsp_status launch_sddmm(const bsp_sddmm_plan* p, const bsp_bsr_desc* mask, const void* A,
                        int64_t lda, const void* B, int64_t ldb, void* out, cudaStream_t stream) {
  if (p->variant == 1) return launch_sddmm_rowstack(p, mask, A, lda, B, ldb, out, stream);
  if (p->n_units == 0) return BSP_OK;
  bsp_device* dev = p->dev;
  SddmmKernelParams kp;
  memset(&kp, 0, sizeof(kp));
  const CUtensorMapSwizzle a_swz =
      p->kc == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  bsp_status st = encode_2d(dev, &kp.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, p->K, p->M, lda,
                            p->kc, p->Rs, a_swz);
  if (st != BSP_OK) return st;
  st = encode_2d(dev, &kp.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, p->N, p->K, ldb, 32, p->kc,
                 CU_TENSOR_MAP_SWIZZLE_64B);
  if (st != BSP_OK) return st;
  kp.units = p->d_units;
  kp.cta_begin = p->d_cta_begin;
  kp.mask_vals = static_cast<const uint16_t*>(mask->values);
  kp.out_vals = static_cast<uint16_t*>(out);
  kp.status = dev->d_status;
  kp.timeout_ns = p->timeout_ns;
  kp.R = p->R;
  kp.C = p->C;
  kp.Rs = p->Rs;
  kp.kc = p->kc;
  kp.nkc = static_cast<int32_t>(p->K / p->kc);
  kp.stages = p->stages;
  kp.stage_bytes = p->stage_bytes;
  kp.a_bytes = p->Rs * p->kc * 2;
  kp.a_swizzle_mode = p->kc == 64 ? 2 : 4;
  kp.tmem_cols = p->tmem_cols;
  kp.keep_a = p->keep_a;
  cudaError_t e = cudaFuncSetAttribute(sddmm_bsr_tcgen05,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, p->smem_bytes);
  if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(sddmm)");
  sddmm_bsr_tcgen05<<<p->grid, kThreads, p->smem_bytes, stream>>>(kp);
  return cuda_check(cudaGetLastError(), "sddmm kernel launch");
}

}  // namespace bsp
