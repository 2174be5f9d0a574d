// BSR SpMM on sm_100a tensor cores:  C[M x N] = A_bsr[M x K] * B[K x N].
//
// Reference path replaced: the three SpMM planners of
// block_spmm/inc/host_code/ and their Tensix kernels, whose device hot loop is
// block_spmm/kernels/compute/bmm_iter.cpp:92-185 (sum over a block-row's
// nonzero blocks of A_blk * B_slice into the DST register).
//
// Mapping ("swap AB"): a 32x32 A block is too short for the 128-row MMA, and
// different block-rows need different B slices, so each CTA computes the
// TRANSPOSED output tile  C_tile^T (128 x Rs) = B_slice^T (128 x C) * A_blk^T:
//   MMA M = 128 dense columns of C (operand A of the MMA = B slice, MN-major,
//           staged by TMA with 128B swizzle: two 64-column boxes),
//   MMA N = Rs rows of the block-row (operand B of the MMA = the A block,
//           K-major, its rows straight out of the BSR value array),
//   MMA K = C, in chunks of kc (64 or 32) per pipeline stage, 16 per MMA.
// Accumulators live in TMEM (fp32), 128 lanes x Rs columns per (n-tile,row).
//
// Work unit = a group of G consecutive block-rows x NT 128-column tiles.  Its
// steps walk the distinct columns of the group: one B slice load per step per
// tile serves every member row with a block in that column (DDA), and one A
// block load serves all NT tiles (SNF).  NAIVE is G = NT = 1.
//
// Warp roles (192 threads, one CTA per SM, persistent over its unit list):
//   warp 0     TMA producer (one thread)
//   warp 1     TMEM allocator + MMA issuer (one thread)
//   warps 2..5 epilogue: tcgen05.ld -> bf16/f32 -> smem -> TMA store; the four
//              warps cover the four 32-lane quarters of TMEM.
// Accumulators are double-buffered so the epilogue of one unit overlaps the
// MMAs of the next.  Every wait is bounded (see bsp_ptx.cuh).
#include <cuda_bf16.h>

#include "bsp_internal.h"
#include "bsp_ptx.cuh"

namespace bsp {
using namespace dev;

namespace {

constexpr int kThreads = 192;
constexpr int kMaxStages = 32;

struct SpmmSmemHeader {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(SpmmSmemHeader) <= 1024, "header must fit its 1 KiB slot");

__device__ __forceinline__ uint32_t bar_addr(const uint64_t* b) { return smem_u32(b); }

// Wait that ignores the abort flag (used to drain our own async copies/MMAs
// before the CTA exits), still bounded.
__device__ __noinline__ bool drain_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl) {
  int zero = 0;
  WaitCtl c2{&zero, ctl.status, ctl.timeout_ns};
  return mbar_wait_bounded(bar, parity, c2, ST_TIMEOUT_DRAIN);
}

__device__ __forceinline__ void spmm_producer(const SpmmKernelParams& p, SpmmSmemHeader* hdr,
                                              uint32_t stage0, int u_begin, int u_end,
                                              const WaitCtl& ctl) {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t armed = 0, armed_parity = 0;
  const uint32_t a_chunk = static_cast<uint32_t>(p.Rs * p.kc * 2);
  const uint32_t b_half = static_cast<uint32_t>(p.kc * 128);
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    const SpmmUnit un = p.units[u];
#pragma unroll 1
    for (int s = un.step_begin; s < un.step_end; ++s) {
      const int32_t* st = p.steps + static_cast<size_t>(s) * p.step_stride;
      const int col = st[0];
      int present = 0;
#pragma unroll 1
      for (int g = 0; g < un.nrows; ++g) present += (st[1 + g] >= 0);
#pragma unroll 1
      for (int kci = 0; kci < p.nkc; ++kci) {
        if (!mbar_wait_bounded(bar_addr(&hdr->empty[stage]), phase ^ 1u, ctl, ST_TIMEOUT_PRODUCER))
          goto drain;
        {
          const uint32_t sb = stage0 + static_cast<uint32_t>(stage) * p.stage_bytes;
          const uint32_t full = bar_addr(&hdr->full[stage]);
          const uint32_t bytes = static_cast<uint32_t>(un.nt) * 2u * b_half + present * a_chunk;
          mbar_arrive_expect_tx(full, bytes);
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          const int ky = col * p.C + kci * p.kc;
#pragma unroll 1
          for (int t = 0; t < un.nt; ++t) {
            tma_load_2d(sb + t * 2 * b_half, &p.tm_b, un.n0 + t * kTileN, ky, full);
            tma_load_2d(sb + t * 2 * b_half + b_half, &p.tm_b, un.n0 + t * kTileN + 64, ky, full);
          }
#pragma unroll 1
          for (int g = 0; g < un.nrows; ++g) {
            const int blk = st[1 + g];
            if (blk >= 0)
              tma_load_2d(sb + p.b_bytes + g * a_chunk, &p.tm_a, kci * p.kc, blk * p.R + un.r_off,
                          full);
          }
        }
        if (++stage == p.stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  }
drain:
  // TMA copies complete on their own: wait for every stage we armed last.
#pragma unroll 1
  for (int s = 0; s < p.stages; ++s)
    if (armed & (1u << s)) drain_wait(bar_addr(&hdr->full[s]), (armed_parity >> s) & 1u, ctl);
}

__device__ __forceinline__ void spmm_mma(const SpmmKernelParams& p, SpmmSmemHeader* hdr,
                                         uint32_t stage0, uint32_t tmem_base, int u_begin,
                                         int u_end, const WaitCtl& ctl) {
  int stage = 0;
  uint32_t phase = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  const uint32_t idesc = idesc_bf16_f32(128, p.Rs, /*a MN-major*/ 1, /*b K-major*/ 0);
  const uint32_t a_chunk = static_cast<uint32_t>(p.Rs * p.kc * 2);
  const uint32_t b_half = static_cast<uint32_t>(p.kc * 128);
  const uint32_t a_sbo = (p.a_swizzle_mode == 2) ? 1024u : 512u;
  const int ksteps = p.kc / 16;
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    const SpmmUnit un = p.units[u];
    if (!mbar_wait_bounded(bar_addr(&hdr->acc_empty[acc]), acc_phase ^ 1u, ctl, ST_TIMEOUT_MMA))
      goto out;
    tc_fence_after();
    {
      const uint32_t d0 = tmem_base + static_cast<uint32_t>(acc * p.acc_cols);
      uint32_t inited = 0;
#pragma unroll 1
      for (int s = un.step_begin; s < un.step_end; ++s) {
        const int32_t* st = p.steps + static_cast<size_t>(s) * p.step_stride;
#pragma unroll 1
        for (int kci = 0; kci < p.nkc; ++kci) {
          if (!mbar_wait_bounded(bar_addr(&hdr->full[stage]), phase, ctl, ST_TIMEOUT_MMA)) goto out;
          tc_fence_after();
          const uint32_t sb = stage0 + static_cast<uint32_t>(stage) * p.stage_bytes;
#pragma unroll 1
          for (int k = 0; k < ksteps; ++k) {
#pragma unroll 1
            for (int t = 0; t < un.nt; ++t) {
              // B slice, MN-major 128B swizzle: LBO = distance between the two
              // 64-column halves, SBO = 8 k-rows of 128 B; 16 k-rows per MMA.
              const uint64_t adesc =
                  smem_desc(sb + t * 2 * b_half + k * 2048u, b_half, 1024u, 2u);
#pragma unroll 1
              for (int g = 0; g < un.nrows; ++g) {
                if (st[1 + g] < 0) continue;
                // A block chunk, K-major: SBO = 8 rows; 16 k-columns = 32 B.
                const uint64_t bdesc = smem_desc(sb + p.b_bytes + g * a_chunk + k * 32u, 16u,
                                                 a_sbo, static_cast<uint32_t>(p.a_swizzle_mode));
                const int slot = t * p.G + g;
                mma_bf16(d0 + static_cast<uint32_t>(slot * p.Rs), adesc, bdesc, idesc,
                         (inited >> slot) & 1u);
                inited |= 1u << slot;
              }
            }
          }
          mma_commit(bar_addr(&hdr->empty[stage]));  // frees the stage when these MMAs finish
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    mma_commit(bar_addr(&hdr->acc_full[acc]));
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1u;
  }
out:
  // Drain every MMA we issued before TMEM is released.
  mma_commit(bar_addr(&hdr->drain));
  drain_wait(bar_addr(&hdr->drain), 0, ctl);
}

template <bool kF32>
__device__ __forceinline__ void spmm_epilogue(const SpmmKernelParams& p, SpmmSmemHeader* hdr,
                                              uint8_t* gbase, uint32_t base, uint32_t epi0,
                                              uint32_t zero_tile, uint32_t tmem_base, int u_begin,
                                              int u_end, const WaitCtl& ctl, int warp, int lane) {
  constexpr uint32_t kEsz = kF32 ? 4u : 2u;
  constexpr uint32_t kTile = 32u * 32u * kEsz;
  const int q = warp & 3;  // TMEM lane quarter this warp may access
  const uint32_t buf0 = epi0 + static_cast<uint32_t>(warp - 2) * 2u * kTile;
  int sb = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    const SpmmUnit un = p.units[u];
    if (!mbar_wait_bounded(bar_addr(&hdr->acc_full[acc]), acc_phase, ctl, ST_TIMEOUT_EPILOGUE))
      break;
    tc_fence_after();
#pragma unroll 1
    for (int t = 0; t < un.nt; ++t) {
      const int ncol = un.n0 + t * kTileN + q * 32;
      if (ncol >= p.N) continue;
#pragma unroll 1
      for (int g = 0; g < un.nrows; ++g) {
        const bool present = (un.row_mask >> g) & 1;
        const int row_base = (un.row0 + g) * p.R + un.r_off;
#pragma unroll 1
        for (int rc = 0; rc < p.Rs / 32; ++rc) {
          uint32_t src = zero_tile;
          if (present) {
            uint32_t v[32];
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * p.acc_cols +
                                                         (t * p.G + g) * p.Rs + rc * 32);
            tmem_ld_32x32b_x32(taddr, v);
            tmem_ld_wait();
            const uint32_t buf = buf0 + static_cast<uint32_t>(sb) * kTile;
            if (lane == 0) bulk_wait_group_read<1>();  // the store that last used `buf` has read it
            __syncwarp();
            uint8_t* gp = gbase + (buf - base);
            if constexpr (kF32) {
              uint32_t* o = reinterpret_cast<uint32_t*>(gp);
#pragma unroll
              for (int r = 0; r < 32; ++r) o[r * 32 + lane] = v[r];
            } else {
              __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(gp);
#pragma unroll
              for (int r = 0; r < 32; ++r) o[r * 32 + lane] = __float2bfloat16_rn(__uint_as_float(v[r]));
            }
            fence_proxy_async_smem();
            __syncwarp();
            src = buf;
            sb ^= 1;
          }
          if (lane == 0) {
            tma_store_2d(&p.tm_c, src, ncol, row_base + rc * 32);
            bulk_commit_group();
          }
          __syncwarp();
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_addr(&hdr->acc_empty[acc]));
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1u;
  }
  if (lane == 0) bulk_wait_group<0>();
  __syncwarp();
}

template <bool kF32>
__global__ void __launch_bounds__(kThreads, 1) spmm_bsr_tcgen05(const __grid_constant__ SpmmKernelParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  SpmmSmemHeader* hdr = reinterpret_cast<SpmmSmemHeader*>(gbase);
  constexpr uint32_t kTile = 32u * 32u * (kF32 ? 4u : 2u);
  const uint32_t stage0 = base + 1024u;
  const uint32_t epi0 = stage0 + static_cast<uint32_t>(p.stages) * p.stage_bytes;
  const uint32_t zero_tile = epi0 + 8u * kTile;

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
    tma_prefetch_desc(&p.tm_c);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&hdr->tmem_base), static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish();
  }
  if (warp >= 2) {
    uint32_t* z = reinterpret_cast<uint32_t*>(gbase + (zero_tile - base));
    for (int i = threadIdx.x - 64; i < static_cast<int>(kTile / 4); i += 128) z[i] = 0u;
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = hdr->tmem_base;
  const WaitCtl ctl{&hdr->abort_flag, p.status, p.timeout_ns};

  if (warp == 0) {
    if (lane == 0) spmm_producer(p, hdr, stage0, u_begin, u_end, ctl);
  } else if (warp == 1) {
    if (lane == 0) spmm_mma(p, hdr, stage0, tmem_base, u_begin, u_end, ctl);
  } else {
    spmm_epilogue<kF32>(p, hdr, gbase, base, epi0, zero_tile, tmem_base, u_begin, u_end, ctl, warp,
                        lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
}

}  // namespace

// Dynamic shared memory the SpMM kernel needs for a given stage layout.
int spmm_smem_bytes(int stages, int stage_bytes, bool c_f32) {
  const int tile = 32 * 32 * (c_f32 ? 4 : 2);
  return 1024 /*align slack*/ + 1024 /*header*/ + stages * stage_bytes + 9 * tile;
}

bsp_status launch_spmm(const bsp_spmm_plan* p, const bsp_bsr_desc* A, const void* B, int64_t ldb,
                       void* C, int64_t ldc, cudaStream_t stream) {
  bsp_device* dev = p->dev;
  const bool f32 = p->c_type == BSP_F32;
  const int esz = f32 ? 4 : 2;
  if (p->n_units == 0 || p->M == 0 || p->N == 0) return BSP_OK;
  SpmmKernelParams kp;
  memset(&kp, 0, sizeof(kp));
  bsp_status st;
  const CUtensorMapSwizzle a_swz =
      p->kc == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (p->nnzb > 0) {
    st = encode_2d(dev, &kp.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A->values, p->C,
                   static_cast<uint64_t>(p->nnzb) * p->R, p->C, p->kc, p->Rs, a_swz);
  } else {  // never read: describe B so the map is well formed
    st = encode_2d(dev, &kp.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, p->N, p->K, ldb, p->kc,
                   p->Rs, a_swz);
  }
  if (st != BSP_OK) return st;
  st = encode_2d(dev, &kp.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, p->N, p->K, ldb, 64, p->kc,
                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != BSP_OK) return st;
  st = encode_2d(dev, &kp.tm_c,
                 f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, esz, C,
                 p->N, p->M, ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st != BSP_OK) return st;
  kp.units = p->d_units;
  kp.cta_begin = p->d_cta_begin;
  kp.steps = p->d_steps;
  kp.status = dev->d_status;
  kp.timeout_ns = p->timeout_ns;
  kp.R = p->R;
  kp.C = p->C;
  kp.Rs = p->Rs;
  kp.kc = p->kc;
  kp.nkc = p->C / p->kc;
  kp.G = p->G;
  kp.NT = p->NT;
  kp.step_stride = 1 + p->G;
  kp.c_f32 = f32;
  kp.stages = p->stages;
  kp.stage_bytes = p->stage_bytes;
  kp.b_bytes = p->NT * p->kc * 256;
  kp.a_swizzle_mode = p->kc == 64 ? 2 : 4;
  kp.acc_cols = p->NT * p->G * p->Rs;
  kp.tmem_cols = p->tmem_cols;
  kp.N = static_cast<int32_t>(p->N);

  auto kern = f32 ? spmm_bsr_tcgen05<true> : spmm_bsr_tcgen05<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       p->smem_bytes);
  if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(spmm)");
  kern<<<p->grid, kThreads, p->smem_bytes, stream>>>(kp);
  return cuda_check(cudaGetLastError(), "spmm kernel launch");
}

}  // namespace bsp
