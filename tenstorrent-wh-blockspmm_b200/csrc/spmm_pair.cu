// BSR SpMM on sm_100a tensor cores, row-stacked form on CTA pairs (2-SM MMA):
//   C[M x N] = A_bsr[M x K] * B[K x N]     (DDA strategy, default kernel)
//
// Same decomposition as spmm_rowstack.cu -- entries (32-row slabs of
// block-rows) stacked along the MMA M dimension, one dense B slice per
// block-column shared by every stacked entry -- but a work unit spans TWO
// CTAs of a cluster: 2G entries (256 output rows) x 256 columns, one
// tcgen05.mma.cta_group::2 of M = 256, N = 256 per 16-deep k-step.
//   * CTA rank r holds entries r*G .. r*G+G-1 (its 128 TMEM lanes, its
//     stacked A operand in its own shared memory) and B columns
//     n0 + 128 r .. +127 of the slice (its half of the N operand).  Each CTA
//     therefore stages half the B bytes of the single-CTA kernel, and the
//     smem ring is twice as deep.
//   * A slot is loaded when its entry has a block in the step, or when it is
//     absent but still holds an older block: then from a TMA box entirely
//     above the A tensor, which the TMA fills with zeros.  Absent slots that
//     are already zero are skipped (the planner replays each CTA's ring).
//     Every shared-memory write is thus a TMA write (async proxy).
//   * Only the leader (rank 0) waits on the full barriers: both CTAs' TMA
//     loads complete on the leader's barrier, armed by the leader with both
//     CTAs' bytes (its stage descriptor carries the pair's count of loaded
//     slots).  The leader issues the MMAs and commits to the empty and
//     accumulator barriers of both CTAs at once (multicast commit arrive).
//   * Each CTA's epilogue reads its own TMEM lanes and writes its rows of C;
//     the peer's epilogue warps arrive on the leader's acc_empty barrier.
// Warp roles per CTA as in the single-CTA kernel (warp 0 MMA, warps 1..3
// producers, warps 4..7 epilogue); the peer's warp 0 only allocates TMEM.
// Every wait is bounded (bsp_ptx.cuh); the pair meets at a cluster barrier
// before TMEM is freed.
#include <cuda_bf16.h>

#include "rowstack_common.cuh"

namespace bsp {
using namespace dev;
using namespace rs;

namespace {

// Producer warp pw of CTA `rank`: stages pw, pw + nprod, ... of the pair's
// sequence, with this CTA's coordinates (stage list of this CTA).
__device__ __forceinline__ void pr_producer(const SpmmKernelParams& p, RsSmemHeader* hdr, uint32_t stage0,
                                           const WaitCtl& ctl, int pw, int lane, uint32_t rank) {
  const int P = p.nprod;
  const int k_begin = p.cta_stage_begin[blockIdx.x];
  const int n = p.cta_stage_begin[blockIdx.x + 1] - k_begin;
  const uint32_t a_slot = static_cast<uint32_t>(p.Rs * p.kc * 2);
  const uint32_t b_blk = static_cast<uint32_t>(p.kc * 128);  // one 64-column box
  const uint32_t b_half = 2u * b_blk;
  const uint32_t sub_bytes = static_cast<uint32_t>(p.sub_bytes);
  const int G = p.G;
  const uint32_t is0 = (lane == 0 && rank == 0) ? 1u : 0u;
  // lanes 0..7: A slot (sub = lane / 4, entry g = lane % 4); lanes 8..11: B
  // (sub = (lane - 8) / 2, 64-column box h = lane % 2; 3-D boxes use lanes 8, 10)
  const int a_sub = lane >> 2, a_g = lane & 3;
  const int b_sub = (lane - 8) >> 1, b_h = lane & 1;
  int stage = pw;
  uint32_t phase = 0;
  uint32_t armed = 0, armed_parity = 0;
  bool ok = true;
#pragma unroll 1
  for (int k0 = pw; k0 < n && ok; k0 += 32 * P) {
    int4 w0 = make_int4(0, 0, 0, 0), w1 = w0, w2 = w0, w3 = w0;
    const int kl = k0 + lane * P;
    if (kl < n) {
      const int4* e = p.stage_list + 4 * static_cast<size_t>(k_begin + kl);
      w0 = __ldg(e);
      w1 = __ldg(e + 1);
      w2 = __ldg(e + 2);
      w3 = __ldg(e + 3);
    }
    const int cnt = min(32, (n - k0 + P - 1) / P);
#pragma unroll 1
    for (int j = 0; j < cnt; ++j) {
      const uint32_t flags = static_cast<uint32_t>(__shfl_sync(0xffffffffu, w0.x, j));
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->empty[stage]), phase ^ 1u, ctl,
                                                     ST_TIMEOUT_PRODUCER));
      if (!ok) break;
      const int bz = __shfl_sync(0xffffffffu, w0.y, j);
      const int ax = __shfl_sync(0xffffffffu, w0.z, j);
      const int ky0 = __shfl_sync(0xffffffffu, w0.w, j);
      const int ky1 = __shfl_sync(0xffffffffu, w1.x, j);
      int ay[8];
      ay[0] = __shfl_sync(0xffffffffu, w1.y, j);
      ay[1] = __shfl_sync(0xffffffffu, w1.z, j);
      ay[2] = __shfl_sync(0xffffffffu, w1.w, j);
      ay[3] = __shfl_sync(0xffffffffu, w2.x, j);
      ay[4] = __shfl_sync(0xffffffffu, w2.y, j);
      ay[5] = __shfl_sync(0xffffffffu, w2.z, j);
      ay[6] = __shfl_sync(0xffffffffu, w2.w, j);
      ay[7] = __shfl_sync(0xffffffffu, w3.x, j);
      int my_ay = ay[0];
#pragma unroll
      for (int i = 1; i < 8; ++i)
        if (lane == i) my_ay = ay[i];
      const uint32_t sb = stage0 + static_cast<uint32_t>(stage) * p.stage_bytes;
      const uint32_t full_local = baddr(&hdr->full[stage]);
      const uint32_t full = mapa_shared(full_local, 0);
      if (rank == 0 && lane == 0)
        hdr->info[stage] = flags & static_cast<uint32_t>(RS_FIRST | RS_LAST | RS_EMPTY | RS_TWO);
      __syncwarp();
      const uint32_t nsub = (flags & RS_EMPTY) ? 0u : ((flags & RS_TWO) ? 2u : 1u);
      // the leader arms its barrier with both CTAs' bytes: B halves and the
      // pair's loaded slots
      const uint32_t np_pair = (flags >> 16) & 0x1Fu;
      mbar_arrive_expect_tx_pred(full_local, nsub * 2u * b_half + np_pair * a_slot, is0);
      if (nsub > 0) {
        const bool a_on = lane < 8 && a_g < G && static_cast<uint32_t>(a_sub) < nsub && ((flags >> lane) & 1u);
        tma_load_2d_pair_pred(sb + static_cast<uint32_t>(a_sub) * sub_bytes + b_half + a_g * a_slot, &p.tm_a,
                              ax, my_ay, full, a_on ? 1u : 0u);
        const int ky = b_sub ? ky1 : ky0;
        if (p.b3d) {
          const bool b_on = lane >= 8 && lane < 12 && b_h == 0 && static_cast<uint32_t>(b_sub) < nsub;
          tma_load_3d_pair_pred(sb + static_cast<uint32_t>(b_sub) * sub_bytes, &p.tm_b, 0, ky, bz, full,
                                b_on ? 1u : 0u);
        } else {
          const bool b_on = lane >= 8 && lane < 12 && static_cast<uint32_t>(b_sub) < nsub;
          tma_load_2d_pair_pred(sb + static_cast<uint32_t>(b_sub) * sub_bytes + b_h * b_blk, &p.tm_b,
                                bz + b_h * 64, ky, full, b_on ? 1u : 0u);
        }
      }
      armed |= 1u << stage;
      armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
      stage += P;
      if (stage >= p.stages) {
        stage -= p.stages;
        phase ^= 1u;
      }
    }
  }
  // The leader's full barriers count both CTAs' bytes: draining them covers
  // the peer's copies too (the peer waits at the final cluster barrier).
  if (rank == 0 && lane == 0) {
#pragma unroll 1
    for (int s = 0; s < p.stages; ++s)
      if (armed & (1u << s)) rs_drain_wait(baddr(&hdr->full[s]), (armed_parity >> s) & 1u, ctl);
  }
  // Every slot this warp filled is released by the leader's MMA warp with a
  // multicast arrive on this CTA's empty barrier; wait for the last of those
  // arrives, so that none is still in flight towards this CTA's shared
  // memory when the CTA exits (it would land in the next launch's CTA on
  // this SM).
  if (lane == 0) {
#pragma unroll 1
    for (int s = 0; s < p.stages; ++s)
      if (armed & (1u << s)) rs_drain_wait(baddr(&hdr->empty[s]), (armed_parity >> s) & 1u, ctl);
  }
  __syncwarp();
}

// MMA warp of the leader: every lane waits, lane 0 issues (predicated).
template <int kKS>
__device__ __forceinline__ void pr_mma(const SpmmKernelParams& p, RsSmemHeader* hdr, uint32_t stage0,
                                      uint32_t tmem_base, int u_begin, int u_end, const WaitCtl& ctl,
                                      int lane) {
  int stage = 0;
  uint32_t phase = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  int units_left = u_end - u_begin;
  // Per CTA: B half = two 64-column MN-major 128B-swizzle boxes (LBO = one
  // box, SBO = 8 k-rows; a 16-row k-step is 2048 bytes), then the stacked A
  // entries (K-major, SBO = 8 rows; a 16-column k-step is 32 bytes).
  const uint32_t idesc = idesc_bf16_f32(256, kRsN, /*a K-major*/ 0, /*b MN-major*/ 1);
  const uint32_t b_half = static_cast<uint32_t>(2 * p.kc * 128);
  const uint32_t a_sbo = (p.a_swizzle_mode == 2) ? 1024u : 512u;
  const uint64_t adesc0 = smem_desc(stage0 + b_half, 16u, a_sbo, static_cast<uint32_t>(p.a_swizzle_mode));
  const uint64_t bdesc0 = smem_desc(stage0, static_cast<uint32_t>(p.kc * 128), 1024u, 2u);
  const uint32_t stage16 = static_cast<uint32_t>(p.stage_bytes) >> 4;
  const uint32_t sub16 = static_cast<uint32_t>(p.sub_bytes) >> 4;
  const uint32_t full0 = baddr(&hdr->full[0]);
  const uint32_t empty0 = baddr(&hdr->empty[0]);
  uint32_t soff = 0;
  uint32_t d0 = tmem_base;
  const uint32_t is0 = lane == 0 ? 1u : 0u;
#pragma unroll 1
  while (units_left > 0) {
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(full0 + stage * 8, phase, ctl, ST_TIMEOUT_MMA))) break;
    tc_fence_after();
    const uint32_t info = hdr->info[stage];
    const bool first = (info & RS_FIRST) != 0;
    if (first) {
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(baddr(&hdr->acc_empty[acc]), acc_phase ^ 1u, ctl, ST_TIMEOUT_MMA)))
        break;
      tc_fence_after();
      d0 = tmem_base + static_cast<uint32_t>(acc * kRsN);
    }
    if (!(info & RS_EMPTY)) {
      const uint64_t ad = adesc0 + soff, bd = bdesc0 + soff;
#pragma unroll
      for (int k = 0; k < kKS; ++k)
        mma_bf16_pair_pred(d0, ad + k * 2u, bd + k * 128u, idesc, (k > 0 || !first) ? 1u : 0u, is0);
      if (info & RS_TWO) {
#pragma unroll
        for (int k = 0; k < kKS; ++k)
          mma_bf16_pair_pred(d0, ad + sub16 + k * 2u, bd + sub16 + k * 128u, idesc, 1u, is0);
      }
      mma_commit_pair_both_pred(empty0 + stage * 8, is0);
      if (info & RS_LAST) mma_commit_pair_both_pred(baddr(&hdr->acc_full[acc]), is0);
    } else if (lane == 0) {
      // A stage (and unit) without blocks has nothing in shared memory and
      // nothing in TMEM to wait for: release it with plain arrives on both
      // CTAs' barriers.  A 2-SM commit is not used here -- with no pair MMA
      // issued before it (a pair whose first units are empty) its multicast
      // arrive was not reliably delivered on B200.
      const uint32_t e_local = empty0 + stage * 8;
      mbar_arrive(e_local);
      mbar_remote_arrive(mapa_shared(e_local, 1));
      if (info & RS_LAST) {
        const uint32_t f_local = baddr(&hdr->acc_full[acc]);
        mbar_arrive(f_local);
        mbar_remote_arrive(mapa_shared(f_local, 1));
      }
    }
    __syncwarp();
    if (info & RS_LAST) {
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
  if (lane == 0) {
    mma_commit_pair_local(baddr(&hdr->drain));
    rs_drain_wait(baddr(&hdr->drain), 0, ctl);
  }
  __syncwarp();
}

template <bool kF32>
__global__ void __launch_bounds__(kRsThreads, 1) spmm_pair_tcgen05(const __grid_constant__ SpmmKernelParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  RsSmemHeader* hdr = reinterpret_cast<RsSmemHeader*>(gbase);
  const uint32_t stage0 = base + 1024u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int u_begin = p.cta_begin[blockIdx.x];
  const int u_end = p.cta_begin[blockIdx.x + 1];
  rs_clear_next_counters(p);

  if (threadIdx.x == 32) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(baddr(&hdr->full[s]), 1);
      mbar_init(baddr(&hdr->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(baddr(&hdr->acc_full[a]), 1);
      mbar_init(baddr(&hdr->acc_empty[a]), 8);  // 4 epilogue warps per CTA of the pair
    }
    mbar_init(baddr(&hdr->drain), 1);
    mbar_init(baddr(&hdr->merge_bar), 4);  // this CTA's epilogue warps (split-K merge)
    hdr->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
  }
  if (warp == kRsMmaWarp) {
    tmem_alloc_pair(smem_u32(&hdr->tmem_base), static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive or copy
  tc_fence_after();
  const uint32_t tmem_base = hdr->tmem_base;
  const WaitCtl ctl{&hdr->abort_flag, p.status, p.timeout_ns};

  if (warp == kRsMmaWarp) {
    if (rank == 0) {
      if (p.kc == 32) pr_mma<2>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
      else pr_mma<4>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
    }
  } else if (warp < kRsEpi0) {
    if (warp - kRsProd0 < p.nprod) pr_producer(p, hdr, stage0, ctl, warp - kRsProd0, lane, rank);
  } else {
    const uint32_t leader_acc_empty = rank == 0 ? 0u : mapa_shared(baddr(&hdr->acc_empty[0]), 0);
    rs_epilogue<kF32>(p, hdr, tmem_base, u_begin, u_end, ctl, warp, lane, leader_acc_empty);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs into this CTA's TMEM are done before it is freed
  if (warp == kRsMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
}

// ---- twin units (variant 3) ---------------------------------------------------
// Two pair units of one column tile share every B slice: a stage is one
// block-column (this CTA's B half, then unit a's four entry slots, then unit
// b's); each unit multiplies into its own accumulator (TMEM columns 0-255 /
// 256-511) at the columns where it holds a block.  One B load thus serves up
// to twice the MMA work of a plain pair stage in the same shared memory.

// Producer warp pw of CTA `rank`: stages pw, pw + nprod, ... of the twin sequence.
__device__ __forceinline__ void tw_producer(const SpmmKernelParams& p, RsSmemHeader* hdr, uint32_t stage0,
                                           const WaitCtl& ctl, int pw, int lane, uint32_t rank) {
  const int P = p.nprod;
  const int k_begin = p.cta_stage_begin[blockIdx.x];
  const int n = p.cta_stage_begin[blockIdx.x + 1] - k_begin;
  const uint32_t a_slot = static_cast<uint32_t>(p.Rs * p.kc * 2);
  const uint32_t b_half = static_cast<uint32_t>(2 * p.kc * 128);
  const uint32_t is0 = (lane == 0 && rank == 0) ? 1u : 0u;
  int stage = pw;
  uint32_t phase = 0;
  uint32_t armed = 0, armed_parity = 0;
  bool ok = true;
#pragma unroll 1
  for (int k0 = pw; k0 < n && ok; k0 += 32 * P) {
    int4 w0 = make_int4(0, 0, 0, 0), w1 = w0, w2 = w0;
    const int kl = k0 + lane * P;
    if (kl < n) {
      const int4* e = p.stage_list + 4 * static_cast<size_t>(k_begin + kl);
      w0 = __ldg(e);
      w1 = __ldg(e + 1);
      w2 = __ldg(e + 2);
    }
    const int cnt = min(32, (n - k0 + P - 1) / P);
#pragma unroll 1
    for (int j = 0; j < cnt; ++j) {
      const uint32_t flags = static_cast<uint32_t>(__shfl_sync(0xffffffffu, w0.x, j));
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->empty[stage]), phase ^ 1u, ctl,
                                                     ST_TIMEOUT_PRODUCER));
      if (!ok) break;
      const int bz = __shfl_sync(0xffffffffu, w0.y, j);
      const int ky = __shfl_sync(0xffffffffu, w0.w, j);
      int ay = __shfl_sync(0xffffffffu, w1.x, j);  // slots 0..7 from w1.x .. w2.w
      const int a1 = __shfl_sync(0xffffffffu, w1.y, j);
      const int a2 = __shfl_sync(0xffffffffu, w1.z, j);
      const int a3 = __shfl_sync(0xffffffffu, w1.w, j);
      const int a4 = __shfl_sync(0xffffffffu, w2.x, j);
      const int a5 = __shfl_sync(0xffffffffu, w2.y, j);
      const int a6 = __shfl_sync(0xffffffffu, w2.z, j);
      const int a7 = __shfl_sync(0xffffffffu, w2.w, j);
      ay = lane == 1 ? a1 : lane == 2 ? a2 : lane == 3 ? a3 : lane == 4 ? a4 : lane == 5 ? a5 : lane == 6 ? a6
           : lane == 7 ? a7 : ay;
      const uint32_t sb = stage0 + static_cast<uint32_t>(stage) * p.stage_bytes;
      const uint32_t full_local = baddr(&hdr->full[stage]);
      const uint32_t full = mapa_shared(full_local, 0);
      if (rank == 0 && lane == 0) hdr->info[stage] = flags;
      __syncwarp();
      const uint32_t loads = (flags & TW_F_EMPTY) ? 0u : (flags & 0xFFu);
      // bytes both CTAs land on the leader's full barrier (the same slot
      // pattern in both: a unit multiplies, or not, on both halves)
      const uint32_t tx = (flags & TW_F_EMPTY) ? 0u : 2u * (b_half + static_cast<uint32_t>(__popc(loads)) * a_slot);
      mbar_arrive_expect_tx_pred(full_local, tx, is0);
      if (!(flags & TW_F_EMPTY)) {
        const bool a_on = lane < 8 && ((loads >> lane) & 1u);
        tma_load_2d_pair_pred(sb + b_half + static_cast<uint32_t>(lane & 7) * a_slot, &p.tm_a, 0, ay, full,
                              a_on ? 1u : 0u);
        if (p.b3d) {
          tma_load_3d_pair_pred(sb, &p.tm_b, 0, ky, bz, full, lane == 8 ? 1u : 0u);
        } else {
          const bool b_on = lane == 8 || lane == 9;
          tma_load_2d_pair_pred(sb + static_cast<uint32_t>(lane & 1) * (b_half / 2), &p.tm_b, bz + (lane & 1) * 64, ky,
                                full, b_on ? 1u : 0u);
        }
      }
      armed |= 1u << stage;
      armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
      stage += P;
      if (stage >= p.stages) {
        stage -= p.stages;
        phase ^= 1u;
      }
    }
  }
  if (rank == 0 && lane == 0) {
#pragma unroll 1
    for (int s = 0; s < p.stages; ++s)
      if (armed & (1u << s)) rs_drain_wait(baddr(&hdr->full[s]), (armed_parity >> s) & 1u, ctl);
  }
  if (lane == 0) {
#pragma unroll 1
    for (int s = 0; s < p.stages; ++s)
      if (armed & (1u << s)) rs_drain_wait(baddr(&hdr->empty[s]), (armed_parity >> s) & 1u, ctl);
  }
  __syncwarp();
}

// MMA warp of the leader: for each stage, each unit that multiplies there
// issues its two k-steps into its accumulator; the stage is released by one
// commit (both CTAs) when any MMA was issued, by plain arrives otherwise.
__device__ __forceinline__ void tw_mma(const SpmmKernelParams& p, RsSmemHeader* hdr, uint32_t stage0,
                                      uint32_t tmem_base, int n_units, const WaitCtl& ctl, int lane) {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t acc_phase[2] = {0u, 0u};
  bool started[2] = {false, false};
  bool any_mma[2] = {false, false};
  int units_left = n_units;
  const uint32_t idesc = idesc_bf16_f32(256, kRsN, /*a K-major*/ 0, /*b MN-major*/ 1);
  const uint32_t b_half = static_cast<uint32_t>(2 * p.kc * 128);
  const uint32_t a_slot = static_cast<uint32_t>(p.Rs * p.kc * 2);
  const uint32_t a_sbo = (p.a_swizzle_mode == 2) ? 1024u : 512u;
  const uint64_t adesc0 = smem_desc(stage0 + b_half, 16u, a_sbo, static_cast<uint32_t>(p.a_swizzle_mode));
  const uint64_t bdesc0 = smem_desc(stage0, static_cast<uint32_t>(p.kc * 128), 1024u, 2u);
  const uint32_t stage16 = static_cast<uint32_t>(p.stage_bytes) >> 4;
  const uint32_t unit16 = (4u * a_slot) >> 4;  // unit b's slots follow unit a's
  const uint32_t full0 = baddr(&hdr->full[0]);
  const uint32_t empty0 = baddr(&hdr->empty[0]);
  uint32_t soff = 0;
  const uint32_t is0 = lane == 0 ? 1u : 0u;
#pragma unroll 1
  while (units_left > 0) {
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(full0 + stage * 8, phase, ctl, ST_TIMEOUT_MMA))) break;
    tc_fence_after();
    const uint32_t info = hdr->info[stage];
    bool ok = true;
    bool issued = false;
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      if (info & (x ? TW_F_FIRST_B : TW_F_FIRST_A)) {
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->acc_empty[x]), acc_phase[x] ^ 1u, ctl,
                                                       ST_TIMEOUT_MMA));
        if (!ok) break;
        tc_fence_after();
        started[x] = false;
        any_mma[x] = false;
      }
      if (info & (x ? TW_F_MMA_B : TW_F_MMA_A)) {
        const uint64_t ad = adesc0 + soff + static_cast<uint32_t>(x) * unit16, bd = bdesc0 + soff;
        const uint32_t d = tmem_base + static_cast<uint32_t>(x * kRsN);
        mma_bf16_pair_pred(d, ad, bd, idesc, started[x] ? 1u : 0u, is0);
        mma_bf16_pair_pred(d, ad + 2u, bd + 128u, idesc, 1u, is0);
        started[x] = true;
        any_mma[x] = true;
        issued = true;
      }
    }
    if (!ok) break;
    if (issued) {
      mma_commit_pair_both_pred(empty0 + stage * 8, is0);
    } else if (lane == 0) {
      // nothing multiplied (an empty twin): plain arrives on both CTAs
      const uint32_t e_local = empty0 + stage * 8;
      mbar_arrive(e_local);
      mbar_remote_arrive(mapa_shared(e_local, 1));
    }
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      if (!(info & (x ? TW_F_LAST_B : TW_F_LAST_A))) continue;
      const uint32_t f_local = baddr(&hdr->acc_full[x]);
      if (any_mma[x]) {
        mma_commit_pair_both_pred(f_local, is0);
      } else if (lane == 0) {
        // a unit without blocks: its accumulator is not read (zero rows)
        mbar_arrive(f_local);
        mbar_remote_arrive(mapa_shared(f_local, 1));
      }
      acc_phase[x] ^= 1u;
      --units_left;
    }
    __syncwarp();
    soff += stage16;
    if (++stage == p.stages) {
      stage = 0;
      soff = 0;
      phase ^= 1u;
    }
  }
  if (lane == 0) {
    mma_commit_pair_local(baddr(&hdr->drain));
    rs_drain_wait(baddr(&hdr->drain), 0, ctl);
  }
  __syncwarp();
}

template <bool kF32>
__global__ void __launch_bounds__(kRsThreads, 1) spmm_twin_tcgen05(const __grid_constant__ SpmmKernelParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  RsSmemHeader* hdr = reinterpret_cast<RsSmemHeader*>(gbase);
  const uint32_t stage0 = base + 1024u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int u_begin = p.cta_begin[blockIdx.x];
  const int u_end = p.cta_begin[blockIdx.x + 1];

  if (threadIdx.x == 32) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(baddr(&hdr->full[s]), 1);
      mbar_init(baddr(&hdr->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(baddr(&hdr->acc_full[a]), 1);
      mbar_init(baddr(&hdr->acc_empty[a]), 8);  // 4 epilogue warps per CTA of the pair
    }
    mbar_init(baddr(&hdr->drain), 1);
    mbar_init(baddr(&hdr->merge_bar), 4);
    hdr->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
  }
  if (warp == kRsMmaWarp) {
    tmem_alloc_pair(smem_u32(&hdr->tmem_base), static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive or copy
  tc_fence_after();
  const uint32_t tmem_base = hdr->tmem_base;
  const WaitCtl ctl{&hdr->abort_flag, p.status, p.timeout_ns};

  if (warp == kRsMmaWarp) {
    if (rank == 0) tw_mma(p, hdr, stage0, tmem_base, u_end - u_begin, ctl, lane);
  } else if (warp < kRsEpi0) {
    if (warp - kRsProd0 < p.nprod) tw_producer(p, hdr, stage0, ctl, warp - kRsProd0, lane, rank);
  } else {
    const uint32_t leader_acc_empty = rank == 0 ? 0u : mapa_shared(baddr(&hdr->acc_empty[0]), 0);
    rs_epilogue<kF32>(p, hdr, tmem_base, u_begin, u_end, ctl, warp, lane, leader_acc_empty);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs into this CTA's TMEM are done before it is freed
  if (warp == kRsMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
}

}  // namespace

bsp_status launch_spmm_pair(const bsp_spmm_plan* p, const bsp_bsr_desc* A, const void* B, int64_t ldb,
                            void* C, int64_t ldc, cudaStream_t stream, void* const* peer_c, int n_peers) {
  bsp_device* dev = p->dev;
  const bool f32 = p->c_type == BSP_F32;
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && !peer_c))
    return set_error(BSP_ERR_INVALID_ARG, "n_peers must be 0..7 with a peer pointer each");
  for (int i = 0; i < n_peers; ++i)
    if (!peer_c[i] || reinterpret_cast<uintptr_t>(peer_c[i]) % 16)
      return set_error(BSP_ERR_INVALID_ARG, "peer C pointers must be non-null and 16-byte aligned");
  if (p->n_units == 0 || p->M == 0 || p->N == 0) return BSP_OK;
  if (reinterpret_cast<uintptr_t>(C) % 16 || (ldc * (f32 ? 4 : 2)) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "C must be 16-byte aligned with 16-byte row pitch");
  if (p->grid % 2) return set_error(BSP_ERR_STATE, "CTA-pair plan with an odd grid");
  auto kern = p->variant == 3 ? (f32 ? spmm_twin_tcgen05<true> : spmm_twin_tcgen05<false>)
                              : (f32 ? spmm_pair_tcgen05<true> : spmm_pair_tcgen05<false>);
  if (!p->attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p->smem_bytes);
    if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(spmm pair)");
    p->attr_set = true;
  }
  SpmmKernelParams& kp = p->kp;
  const bool cached = p->kp_valid && p->kp_a == A->values && p->kp_b == B && p->kp_c == C &&
                      p->kp_ldb == ldb && p->kp_ldc == ldc;
  if (!cached) {
    p->kp_valid = false;
    memset(&kp, 0, sizeof(kp));
    bsp_status st;
    const CUtensorMapSwizzle a_swz = p->kc == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    if (p->nnzb > 0) {
      st = encode_2d(dev, &kp.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A->values, p->C,
                     static_cast<uint64_t>(p->nnzb) * p->R, p->C, p->kc, p->Rs, a_swz);
    } else {
      // no blocks: every A slot is a zero box, any valid map serves
      st = encode_2d(dev, &kp.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, p->N, p->K, ldb, p->kc, p->Rs,
                     a_swz);
    }
    if (st != BSP_OK) return st;
    const bool b3d = (p->N % 64 == 0);
    if (b3d) {
      const uint64_t dims[3] = {64, static_cast<uint64_t>(p->K), static_cast<uint64_t>(p->N / 64)};
      const uint64_t strides[2] = {static_cast<uint64_t>(ldb) * 2, 128};
      const uint32_t box[3] = {64, static_cast<uint32_t>(p->kc), 2};
      st = encode_nd(dev, &kp.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, B, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
      st = encode_2d(dev, &kp.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, p->N, p->K, ldb, 64, p->kc,
                     CU_TENSOR_MAP_SWIZZLE_128B);
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
    kp.NT = 2;
    kp.step_stride = p->step_stride;
    kp.c_f32 = f32;
    kp.stages = p->stages;
    kp.stage_bytes = p->stage_bytes;
    kp.b_bytes = 2 * p->kc * 128;
    kp.a_swizzle_mode = p->kc == 64 ? 2 : 4;
    kp.acc_cols = kRsN;
    kp.stacked = 1;
    kp.tmem_cols = p->tmem_cols;
    kp.N = static_cast<int32_t>(p->N);
    kp.nprod = p->nprod;
    kp.b3d = b3d;
    kp.stage_list = p->d_stage_list;
    kp.cta_stage_begin = p->d_cta_stage_begin;
    kp.sub_bytes = p->sub_bytes;
    kp.xfer_off = p->xfer_off;
    kp.split_ws = p->d_split_ws;
      p->kp_valid = true;
    p->kp_a = A->values;
    p->kp_b = B;
    p->kp_c = C;
    p->kp_ldb = ldb;
    p->kp_ldc = ldc;
  }
  kp.n_peers = n_peers;
  for (int i = 0; i < kMaxPeers; ++i) kp.peer_c[i] = i < n_peers ? peer_c[i] : nullptr;
  select_split_counters(p, kp);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p->grid));
  cfg.blockDim = dim3(kRsThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(p->smem_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, kp);
  if (e != cudaSuccess) return cuda_check(e, "spmm pair kernel launch");
  return cuda_check(cudaGetLastError(), "spmm pair kernel launch");
}

}  // namespace bsp
