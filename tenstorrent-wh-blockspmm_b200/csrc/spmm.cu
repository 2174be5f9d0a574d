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
//           staged by TMA with 128B swizzle as 64-column boxes),
//   MMA N = Rs rows of the block-row (operand B of the MMA = the A block,
//           K-major, its rows straight out of the BSR value array),
//   MMA K = C, in chunks of kc (64 or 32) per pipeline stage, 16 per MMA.
// Accumulators live in TMEM (fp32), 128 lanes x Rs columns per (n-tile,row).
//
// Work unit = a group of G consecutive block-rows x NT 128-column tiles.  Its
// steps walk the distinct columns of the group: one B slice load per step
// serves every member row with a block in that column (DDA), and one A block
// load serves all NT tiles (SNF).  NAIVE is G = NT = 1.  With "stacked" MMAs
// (DDA default) the group's blocks of a step sit side by side in shared memory
// as one K-major operand of G*Rs rows (absent rows zeroed), so each k-step is
// ONE MMA of N = G*Rs instead of one per row.
//
// Warp roles (288 threads, one CTA per SM, persistent over its unit list):
//   warps 0..3  TMA producers: warp w issues every nprod-th pipeline stage, so
//               several threads keep the TMA engine fed (one issuing thread
//               cannot: each TMA instruction costs it ~0.1 us)
//   warp 4      TMEM allocator + MMA issuer (one thread)
//   warps 5..8  epilogue: tcgen05.ld -> bf16/f32 -> direct coalesced global
//               stores; the four warps cover the four 32-lane quarters of TMEM.
// Accumulators are double-buffered so the epilogue of one unit overlaps the
// MMAs of the next.  Every wait is bounded (see bsp_ptx.cuh).
#include <cuda_bf16.h>

#include <type_traits>

#include "bsp_internal.h"
#include "bsp_ptx.cuh"

namespace bsp {
using namespace dev;

namespace {

constexpr int kProducerWarps = 4;
constexpr int kMmaWarp = kProducerWarps;  // warps kMmaWarp+1 .. +4 are the epilogue
constexpr int kThreads = (kProducerWarps + 5) * 32;
constexpr int kMaxStages = 32;

struct SpmmSmemHeader {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t info[kMaxStages];  // per-stage work description, written by the producer
  uint8_t zeroed[kMaxStages];  // per-stage: bit g = A slot g holds zeros
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(SpmmSmemHeader) <= 1024, "header must fit its 1 KiB slot");

// Stage info word (producer -> MMA thread, published by the full barrier).
enum : uint32_t {
  INFO_PRESENT_MASK = 0xFFu,  // bit g: group row g has a block in this step
  INFO_NT_SHIFT = 8,          // bits 8..10: 128-column tiles of the unit
  INFO_FIRST = 1u << 12,      // first stage of a unit
  INFO_LAST = 1u << 13,       // last stage of a unit
  INFO_EMPTY = 1u << 14,      // unit without blocks: no loads, no MMAs
};

__device__ __forceinline__ uint32_t bar_addr(const uint64_t* b) { return smem_u32(b); }

// Wait that ignores the abort flag (used to drain our own async copies/MMAs
// before the CTA exits), still bounded.
__device__ __noinline__ bool drain_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl) {
  int zero = 0;
  WaitCtl c2{&zero, ctl.status, ctl.timeout_ns};
  return mbar_wait_bounded(bar, parity, c2, ST_TIMEOUT_DRAIN);
}

// Producer warp `pw`: walks the whole unit list in step with the other
// producer warps and issues the stages whose sequence number is pw mod nprod.
// Step metadata is fetched 32 steps at a time (one coalesced load per lane,
// broadcast by shuffles).
__device__ __forceinline__ void spmm_producer(const SpmmKernelParams& p, SpmmSmemHeader* hdr,
                                              uint8_t* gbase, uint32_t base, uint32_t stage0,
                                              int u_begin, int u_end, const WaitCtl& ctl, int pw,
                                              int lane) {
  int stage = 0;
  uint32_t phase = 0;
  int rr = 0;  // round-robin position of the current stage among producer warps
  uint32_t armed = 0, armed_parity = 0;
  bool ok = true;
  const uint32_t a_chunk = static_cast<uint32_t>(p.Rs * p.kc * 2);
  const uint32_t b_half = static_cast<uint32_t>(p.kc * 128);
  const int G = p.G;
  const uint32_t b_bytes_full = p.b3d ? static_cast<uint32_t>(p.NT) * 2u * b_half : 0u;
#pragma unroll 1
  for (int u = u_begin; u < u_end && ok; ++u) {
    const SpmmUnit un = p.units[u];
    const int nsteps = un.step_end - un.step_begin;
    const uint32_t nt_bits = static_cast<uint32_t>(un.nt) << INFO_NT_SHIFT;
    if (nsteps == 0) {
      // A unit without blocks still passes through the MMA thread once so the
      // accumulator hand-off stays in order; the epilogue writes zeros.
      if (rr == pw && lane == 0) {
        ok = mbar_wait_bounded(bar_addr(&hdr->empty[stage]), phase ^ 1u, ctl, ST_TIMEOUT_PRODUCER);
        if (ok) {
          hdr->info[stage] = INFO_FIRST | INFO_LAST | INFO_EMPTY | nt_bits;
          mbar_arrive(bar_addr(&hdr->full[stage]));
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (++rr == p.nprod) rr = 0;
      if (++stage == p.stages) {
        stage = 0;
        phase ^= 1u;
      }
      continue;
    }
#pragma unroll 1
    for (int s0 = 0; s0 < nsteps && ok; s0 += 32) {
      int my_col = 0;
      int my_blk[kMaxGroupRows];
#pragma unroll
      for (int g = 0; g < kMaxGroupRows; ++g) my_blk[g] = -1;
      if (s0 + lane < nsteps) {
        const int32_t* st = p.steps + static_cast<size_t>(un.step_begin + s0 + lane) * p.step_stride;
        my_col = __ldg(st);
#pragma unroll
        for (int g = 0; g < kMaxGroupRows; ++g)
          if (g < G) my_blk[g] = __ldg(st + 1 + g);
      }
      const int cnt = min(32, nsteps - s0);
#pragma unroll 1
      for (int j = 0; j < cnt && ok; ++j) {
        const int col = __shfl_sync(0xffffffffu, my_col, j);
        int blk[kMaxGroupRows];
        uint32_t present = 0;
        int npresent = 0;
#pragma unroll
        for (int g = 0; g < kMaxGroupRows; ++g) {
          blk[g] = __shfl_sync(0xffffffffu, my_blk[g], j);
          if (g < un.nrows && blk[g] >= 0) {
            present |= 1u << g;
            ++npresent;
          }
        }
#pragma unroll 1
        for (int kci = 0; kci < p.nkc; ++kci) {
          if (rr == pw) {
            ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_addr(&hdr->empty[stage]), phase ^ 1u, ctl,
                                                           ST_TIMEOUT_PRODUCER));
            if (!ok) break;
            const uint32_t sb = stage0 + static_cast<uint32_t>(stage) * p.stage_bytes;
            if (p.stacked) {
              // absent rows of the stacked operand must read as zeros: clear
              // their slots once (a slot stays zero until a block lands in it)
              const uint32_t need = (~present) & ((1u << G) - 1u) & ~uint32_t(hdr->zeroed[stage]);
              if (need) {
#pragma unroll 1
                for (uint32_t m = need; m; m &= m - 1) {
                  const int g = __ffs(m) - 1;
                  uint4* dst = reinterpret_cast<uint4*>(gbase + (sb + p.b_bytes + g * a_chunk - base));
                  for (uint32_t i = lane; i < a_chunk / 16; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
                }
                fence_proxy_async_smem();
              }
              __syncwarp();
              if (lane == 0) hdr->zeroed[stage] = static_cast<uint8_t>((hdr->zeroed[stage] | need) & ~present);
            }
            if (lane == 0) {
              const uint32_t full = bar_addr(&hdr->full[stage]);
              uint32_t info = present | nt_bits;
              if (s0 + j == 0 && kci == 0) info |= INFO_FIRST;
              if (s0 + j == nsteps - 1 && kci == p.nkc - 1) info |= INFO_LAST;
              hdr->info[stage] = info;
              const uint32_t b_bytes = p.b3d ? b_bytes_full : static_cast<uint32_t>(un.nt) * 2u * b_half;
              mbar_arrive_expect_tx(full, b_bytes + static_cast<uint32_t>(npresent) * a_chunk);
              armed |= 1u << stage;
              armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
              const int ky = col * p.C + kci * p.kc;
              if (p.b3d) {
                // one box: 2*NT column blocks of 64 x kc rows
                tma_load_3d(sb, &p.tm_b, 0, ky, un.n0 / 64, full);
              } else {
#pragma unroll 1
                for (int t = 0; t < un.nt; ++t) {
                  tma_load_2d(sb + t * 2 * b_half, &p.tm_b, un.n0 + t * kTileN, ky, full);
                  tma_load_2d(sb + t * 2 * b_half + b_half, &p.tm_b, un.n0 + t * kTileN + 64, ky, full);
                }
              }
#pragma unroll
              for (int g = 0; g < kMaxGroupRows; ++g)
                if ((present >> g) & 1u)
                  tma_load_2d(sb + p.b_bytes + g * a_chunk, &p.tm_a, kci * p.kc,
                              blk[g] * p.R + un.r_off, full);
            }
          }
          if (++rr == p.nprod) rr = 0;
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  }
  if (lane == 0) {
    // TMA copies complete on their own: wait for every stage we armed last.
#pragma unroll 1
    for (int s = 0; s < p.stages; ++s)
      if (armed & (1u << s)) drain_wait(bar_addr(&hdr->full[s]), (armed_parity >> s) & 1u, ctl);
  }
  __syncwarp();
}

// MMA issuer: consumes stages in order, driven only by the stage info words
// in shared memory.  The whole warp runs the loop without diverging: every
// lane waits on the barriers and executes the MMA and commit instructions
// predicated on lane 0 (a lone issuing lane costs hundreds of cycles per
// stage in divergent-warp scheduling).  The issuing lane's instruction latency
// bounds the kernel, so the loop is kept lean: k-steps per stage are a
// template constant, descriptors are stage-0 templates moved by precomputed
// 16-byte offsets, and stacked operands need one MMA per (k-step, tile).
template <int kKS, bool kStacked>
__device__ __forceinline__ void spmm_mma(const SpmmKernelParams& p, SpmmSmemHeader* hdr,
                                         uint32_t stage0, uint32_t tmem_base, int u_begin,
                                         int u_end, const WaitCtl& ctl, int lane) {
  int stage = 0;
  uint32_t phase = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  int units_left = u_end - u_begin;
  const uint32_t idesc_row = idesc_bf16_f32(128, p.Rs, /*a MN-major*/ 1, /*b K-major*/ 0);
  const uint32_t idesc_grp = idesc_bf16_f32(128, p.G * p.Rs, 1, 0);
  const uint32_t a_chunk16 = static_cast<uint32_t>(p.Rs * p.kc * 2) >> 4;
  const uint32_t b_half = static_cast<uint32_t>(p.kc * 128);
  const uint32_t tile16 = (2u * b_half) >> 4;  // one 128-column tile of the B slice
  const uint32_t a_sbo = (p.a_swizzle_mode == 2) ? 1024u : 512u;
  // Descriptor templates for stage 0; a byte offset d moves them by d >> 4.
  // B slice: MN-major 128B swizzle, LBO = one 64-column block, SBO = 8 k-rows;
  // a 16-row k-step is 2048 bytes.
  const uint64_t bdesc0 = smem_desc(stage0, b_half, 1024u, 2u);
  // A blocks: K-major, SBO = 8 rows; a 16-column k-step is 32 bytes.
  const uint64_t adesc0 = smem_desc(stage0 + p.b_bytes, 16u, a_sbo, static_cast<uint32_t>(p.a_swizzle_mode));
  const uint32_t stage16 = static_cast<uint32_t>(p.stage_bytes) >> 4;
  const uint32_t grp_cols = static_cast<uint32_t>(p.G * p.Rs);
  const uint32_t full0 = bar_addr(&hdr->full[0]);
  const uint32_t empty0 = bar_addr(&hdr->empty[0]);
  uint32_t soff = 0;
  uint32_t d0 = tmem_base;
  uint32_t inited = 0;
  const uint32_t is0 = lane == 0 ? 1u : 0u;
#pragma unroll 1
  while (units_left > 0) {
    // lanes agree on every wait's outcome, so a timeout leaves the loop warp-wide
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(full0 + stage * 8, phase, ctl, ST_TIMEOUT_MMA))) break;
    const uint32_t info = hdr->info[stage];
    const bool first = (info & INFO_FIRST) != 0;
    if (first) {
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(bar_addr(&hdr->acc_empty[acc]), acc_phase ^ 1u, ctl, ST_TIMEOUT_MMA)))
        break;
      d0 = tmem_base + static_cast<uint32_t>(acc * p.acc_cols);
      inited = 0;
    }
    tc_fence_after();
    if (!(info & INFO_EMPTY)) {
      const int nt = static_cast<int>((info >> INFO_NT_SHIFT) & 7u);
      const uint64_t bd_s = bdesc0 + soff;
      const uint64_t ad_s = adesc0 + soff;
      if constexpr (kStacked) {
        // every tile's accumulator starts at the unit's first stage, k = 0
#pragma unroll
        for (int k = 0; k < kKS; ++k)
#pragma unroll
          for (int t = 0; t < kMaxNTiles; ++t)
            if (t < nt)
              mma_bf16_pred(d0 + t * grp_cols, bd_s + t * tile16 + k * 128u, ad_s + k * 2u, idesc_grp,
                            (k > 0 || !first) ? 1u : 0u, is0);
      } else {
        const uint32_t present = info & INFO_PRESENT_MASK;
#pragma unroll
        for (int k = 0; k < kKS; ++k) {
#pragma unroll 1
          for (int t = 0; t < nt; ++t) {
#pragma unroll 1
            for (uint32_t m = present; m; m &= m - 1) {
              const int g = __ffs(m) - 1;
              const int slot = t * p.G + g;
              mma_bf16_pred(d0 + static_cast<uint32_t>(slot * p.Rs), bd_s + t * tile16 + k * 128u,
                            ad_s + g * a_chunk16 + k * 2u, idesc_row, (inited >> slot) & 1u, is0);
              inited |= 1u << slot;
            }
          }
        }
      }
    }
    mma_commit_pred(empty0 + stage * 8, is0);  // frees the stage when these MMAs finish
    if (info & INFO_LAST) {
      mma_commit_pred(bar_addr(&hdr->acc_full[acc]), is0);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      --units_left;
    }
    soff += stage16;
    if (++stage == p.stages) {
      stage = 0;
      soff = 0;
      phase ^= 1u;
    }
  }
  // Drain every MMA we issued before TMEM is released.
  if (lane == 0) {
    mma_commit(bar_addr(&hdr->drain));
    drain_wait(bar_addr(&hdr->drain), 0, ctl);
  }
  __syncwarp();
}

// Epilogue warp: TMEM lane quarter q holds output columns n0 + 32q + lane of
// every (tile, row) accumulator; each tcgen05.ld gives a thread 32 rows of its
// column, written straight to C (a warp writes 32 consecutive columns of a row
// per store instruction).
template <bool kF32>
__device__ __forceinline__ void spmm_epilogue(const SpmmKernelParams& p, SpmmSmemHeader* hdr,
                                              uint32_t tmem_base, int u_begin, int u_end,
                                              const WaitCtl& ctl, int warp, int lane) {
  using Out = typename std::conditional<kF32, float, __nv_bfloat16>::type;
  const int q = warp & 3;
  int acc = 0;
  uint32_t acc_phase = 0;
  Out* const C = static_cast<Out*>(p.c_ptr);
  const int64_t ldc = p.ldc;
  SpmmUnit nxt;
  if (u_begin < u_end) nxt = p.units[u_begin];
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    const SpmmUnit un = nxt;
    if (u + 1 < u_end) nxt = p.units[u + 1];  // prefetch while this unit's MMAs run
    if (!mbar_wait_bounded(bar_addr(&hdr->acc_full[acc]), acc_phase, ctl, ST_TIMEOUT_EPILOGUE))
      break;
    tc_fence_after();
#pragma unroll 1
    for (int t = 0; t < un.nt; ++t) {
      const int nbase = un.n0 + t * kTileN + q * 32;
      if (nbase >= p.N) continue;
      const int n = nbase + lane;
      const bool col_ok = n < p.N;
#pragma unroll 1
      for (int g = 0; g < un.nrows; ++g) {
        const bool present = (un.row_mask >> g) & 1;
        const int64_t row_base = static_cast<int64_t>(un.row0 + g) * p.R + un.r_off;
#pragma unroll 1
        for (int rc = 0; rc < p.Rs / 32; ++rc) {
          Out* dst = C + (row_base + rc * 32) * ldc + n;
          if (present) {
            uint32_t v[32];
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * p.acc_cols +
                                                         (t * p.G + g) * p.Rs + rc * 32);
            tmem_ld_32x32b_x32(taddr, v);
            tmem_ld_wait();
            if (col_ok) {
#pragma unroll
              for (int r = 0; r < 32; ++r) {
                if constexpr (kF32)
                  dst[r * ldc] = __uint_as_float(v[r]);
                else
                  dst[r * ldc] = __float2bfloat16_rn(__uint_as_float(v[r]));
              }
            }
          } else if (col_ok) {
#pragma unroll
            for (int r = 0; r < 32; ++r) dst[r * ldc] = Out(0.0f);
          }
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

template <bool kF32>
__global__ void __launch_bounds__(kThreads, 1) spmm_bsr_tcgen05(const __grid_constant__ SpmmKernelParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  SpmmSmemHeader* hdr = reinterpret_cast<SpmmSmemHeader*>(gbase);
  const uint32_t stage0 = base + 1024u;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int u_begin = p.cta_begin[blockIdx.x];
  const int u_end = p.cta_begin[blockIdx.x + 1];

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(bar_addr(&hdr->full[s]), 1);
      mbar_init(bar_addr(&hdr->empty[s]), 1);
      hdr->zeroed[s] = 0;
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
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&hdr->tmem_base), static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = hdr->tmem_base;
  const WaitCtl ctl{&hdr->abort_flag, p.status, p.timeout_ns};

  if (warp < kProducerWarps) {
    if (warp < p.nprod)
      spmm_producer(p, hdr, gbase, base, stage0, u_begin, u_end, ctl, warp, lane);
  } else if (warp == kMmaWarp) {
    if (p.kc == 32) {
      if (p.stacked) spmm_mma<2, true>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
      else spmm_mma<2, false>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
    } else {
      if (p.stacked) spmm_mma<4, true>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
      else spmm_mma<4, false>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
    }
  } else {
    spmm_epilogue<kF32>(p, hdr, tmem_base, u_begin, u_end, ctl, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
}

}  // namespace

int spmm_threads() { return kThreads; }
int spmm_max_producers() { return kProducerWarps; }

// Dynamic shared memory the SpMM kernel needs for a given stage layout.
int spmm_smem_bytes(int stages, int stage_bytes, bool /*c_f32*/) {
  return 1024 /*align slack*/ + 1024 /*header*/ + stages * stage_bytes;
}

bsp_status launch_spmm(const bsp_spmm_plan* p, const bsp_bsr_desc* A, const void* B, int64_t ldb,
                       void* C, int64_t ldc, cudaStream_t stream) {
  bsp_device* dev = p->dev;
  const bool f32 = p->c_type == BSP_F32;
  if (p->n_units == 0 || p->M == 0 || p->N == 0) return BSP_OK;
  if (reinterpret_cast<uintptr_t>(C) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "C must be 16-byte aligned");
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
  // B: a 3-D view (64 columns, K rows, 64-column blocks) lets one box carry all
  // of a unit's tiles; it needs every block to lie inside B's rows.
  const bool b3d = (p->N % 64 == 0);
  if (b3d) {
    const uint64_t dims[3] = {64, static_cast<uint64_t>(p->K), static_cast<uint64_t>(p->N / 64)};
    const uint64_t strides[2] = {static_cast<uint64_t>(ldb) * 2, 128};
    const uint32_t box[3] = {64, static_cast<uint32_t>(p->kc), static_cast<uint32_t>(2 * p->NT)};
    st = encode_nd(dev, &kp.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, B, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    st = encode_2d(dev, &kp.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, p->N, p->K, ldb, 64,
                   p->kc, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (st != BSP_OK) return st;
  kp.units = p->d_units;
  kp.cta_begin = p->d_cta_begin;
  kp.steps = p->d_steps;
  kp.status = dev->d_status;
  kp.timeout_ns = p->timeout_ns;
  kp.c_ptr = C;
  kp.ldc = ldc;
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
  kp.stacked = p->stacked;
  kp.tmem_cols = p->tmem_cols;
  kp.N = static_cast<int32_t>(p->N);
  kp.nprod = p->nprod;
  kp.b3d = b3d;

  auto kern = f32 ? spmm_bsr_tcgen05<true> : spmm_bsr_tcgen05<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       p->smem_bytes);
  if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(spmm)");
  kern<<<p->grid, kThreads, p->smem_bytes, stream>>>(kp);
  return cuda_check(cudaGetLastError(), "spmm kernel launch");
}

}  // namespace bsp
