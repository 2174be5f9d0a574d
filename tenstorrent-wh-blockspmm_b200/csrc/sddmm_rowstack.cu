// BSR SDDMM on sm_100a tensor cores, row-stacked form:
//   out(i, j) = mask(i, j) (.) (A[iR:(i+1)R, :] * B[:, jC:(j+1)C])   for every mask block (i, j).
//
// Reference path replaced: block_sddmm/inc/host_code/bsr_sddmm_multicore_{naive,CDA}.cpp
// and their Tensix kernels; device hot loop block_sddmm/kernels/compute/
// sddmm_block_multiply.cpp:72-193 (matmul over K steps, Hadamard with the mask).
//
// Mapping: a work unit is 128 consecutive output rows (MMA M; one TMA box of
// A, four 32-row slabs = the four TMEM lane quarters) against up to eight
// 32-column segments of B gathered from the mask's block-columns of those
// rows (MMA N = 32 * nseg_max = 128 or 256, MN-major with 64B swizzle, one
// TMA box per segment).  K runs in kc-wide pipeline stages (kc/16 MMAs
// each).  The fp32 accumulator sits in TMEM, double-buffered; the epilogue
// writes the (slab, segment) tiles that the mask holds, multiplied by the
// mask value in fp32 and rounded once to bf16, into the mask's block layout.
// The rows of A are shared by every segment of the unit, the way the
// reference's CDA keeps the A row resident while B blocks stream past.
// Resident-A form (keep_a; the CDA and SnF strategies): the 128 x K A tile of
// a row group is loaded once into one of two A buffers and kept while the
// CTA's consecutive units of that group run, so the pipeline stages carry B
// segments only (the L2 -> SM fill, not the MMA, bounds this kernel).  The
// planner marks each unit's run of equal row0 (pad[0] = run << 1 | first,
// pad[1] = last).
//
// Warp roles (384 threads, one persistent CTA per SM):
//   warp 0      TMEM allocator + MMA issuer (warp-converged, lane 0 issues)
//   warps 1..3  TMA producers: warp w owns the ring slots congruent to it; one
//               predicated instruction issues the A box and every segment box
//               of a stage (lane 8: A, lanes 0..nseg-1: the segments)
//   warps 4..11 epilogue: TMEM lane quarter q = warp & 3 = slab q; the two
//               warps of a quarter take alternate segments, and each overlaps
//               the TMEM load of its next tile with the stores of the current
// Every wait is bounded (bsp_ptx.cuh).
#include <cuda_bf16.h>

#include "bsp_internal.h"
#include "bsp_ptx.cuh"

namespace bsp {
using namespace dev;

namespace {

constexpr int kSdMmaWarp = 0;
constexpr int kSdProd0 = 1;
constexpr int kSdMaxProducers = 3;
constexpr int kSdEpi0 = 4;
constexpr int kSdEpiWarps = 8;
constexpr int kSdThreads = (kSdEpi0 + kSdEpiWarps) * 32;
constexpr int kSdMaxStages = 30;

struct SdSmemHeader {
  uint64_t full[kSdMaxStages];
  uint64_t empty[kSdMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t a_full[2];   // resident A buffers
  uint64_t a_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int a_ticket;         // resident A: the next run whose tile may be issued
};
static_assert(sizeof(SdSmemHeader) <= 1024, "header must fit its 1 KiB slot");

__device__ __forceinline__ uint32_t baddr(const uint64_t* b) { return smem_u32(b); }

__device__ __noinline__ bool sd_drain_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl) {
  int zero = 0;
  WaitCtl c2{&zero, ctl.status, ctl.timeout_ns};
  return mbar_wait_bounded(bar, parity, c2, ST_TIMEOUT_DRAIN);
}

// Resident A: several producer warps issue A tiles, each for the runs whose
// first stage it owns.  A buffer's release is a parity wait, which cannot
// tell phase n from n + 2, so the tiles are issued strictly in run order:
// the loader of run r waits (bounded) until a_ticket == r.
__device__ __noinline__ bool sd_ticket_wait(volatile int* ticket, int want, const WaitCtl& ctl) {
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    if (*ticket == want) return true;
    if (*ctl.abort_flag) return false;
    if (globaltimer_ns() - t0 > ctl.timeout_ns) {
      *ctl.abort_flag = 1;
      atomicOr(ctl.status, ST_TIMEOUT_PRODUCER);
      return false;
    }
  }
}

// Word `lane` (< 12) of a unit record: row0, nseg, pad, pad, seg_col[0..7].
__device__ __forceinline__ int32_t unit_word(const SddmmRsUnit* u, int lane) {
  return lane < 12 ? __ldg(reinterpret_cast<const int32_t*>(u) + lane) : 0;
}

// Producer warp pw: stages pw, pw + P, ... of this CTA's sequence (unit-major,
// nkc k-chunks per unit).  The record of the unit of the next owned stage is
// fetched one stage ahead, so the issuing lanes rarely wait on global memory.
// kKeepA: the warp that owns a run's first stage also loads the run's A tile
// (lanes 8.. one k-chunk box each) into A buffer run & 1.
template <bool kKeepA>
__device__ __forceinline__ void sd_producer(const SddmmKernelParams& p, SdSmemHeader* hdr,
                                           uint32_t stage0, uint32_t abuf0, int u_begin, int u_end,
                                           const WaitCtl& ctl, int pw, int lane) {
  const int P = p.nprod;
  const int nkc = p.nkc;
  const int64_t total = static_cast<int64_t>(u_end - u_begin) * nkc;
  const uint32_t a_bytes = static_cast<uint32_t>(p.a_bytes);  // one k-chunk of the 128 rows
  const uint32_t seg_bytes = static_cast<uint32_t>(p.seg_bytes);
  const uint32_t b_off = kKeepA ? 0u : a_bytes;               // B segments' offset in a stage
  int stage = pw;
  uint32_t phase = 0;
  uint32_t armed = 0, armed_parity = 0;
  int cur_u = -1;
  int32_t cur_w = 0;
  int next_u = (pw < total) ? u_begin + pw / nkc : -1;
  int32_t next_w = next_u >= 0 ? unit_word(p.rs_units + next_u, lane) : 0;
#pragma unroll 1
  for (int64_t g = pw; g < total; g += P) {
    const int u = u_begin + static_cast<int>(g / nkc);
    const int kci = static_cast<int>(g % nkc);
    if (u != cur_u) {
      cur_u = u;
      cur_w = (u == next_u) ? next_w : unit_word(p.rs_units + u, lane);
    }
    // prefetch the record of the next owned stage's unit
    const int64_t g2 = g + P;
    const int u2 = g2 < total ? u_begin + static_cast<int>(g2 / nkc) : -1;
    if (u2 >= 0 && u2 != cur_u && u2 != next_u) {
      next_u = u2;
      next_w = unit_word(p.rs_units + u2, lane);
    }
    const int32_t row0 = __shfl_sync(0xffffffffu, cur_w, 0);
    const int32_t nseg = __shfl_sync(0xffffffffu, cur_w, 1);
    const int32_t my_col = __shfl_sync(0xffffffffu, cur_w, 4 + (lane & 7));
    if (kKeepA && kci == 0) {
      const int32_t run = __shfl_sync(0xffffffffu, cur_w, 2);
      if (run & 1) {  // first unit of a run: its A tile into buffer (run >> 1) & 1
        const uint32_t buf = static_cast<uint32_t>(run >> 1) & 1u;
        const uint32_t use = static_cast<uint32_t>(run >> 2) & 1u;  // uses of this buffer so far, mod 2
        if (!__all_sync(0xffffffffu, sd_ticket_wait(&hdr->a_ticket, run >> 1, ctl))) break;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->a_empty[buf]), use ^ 1u, ctl,
                                                        ST_TIMEOUT_PRODUCER)))
          break;
        const uint32_t af = baddr(&hdr->a_full[buf]);
        mbar_arrive_expect_tx_pred(af, a_bytes * static_cast<uint32_t>(nkc), lane == 0);
        const int ch = lane - 8;  // lanes 8 .. 8 + nkc - 1: one k-chunk box each
        tma_load_2d_pred(abuf0 + buf * a_bytes * static_cast<uint32_t>(nkc) + static_cast<uint32_t>(ch & 7) * a_bytes,
                         &p.tm_a, (ch & 7) * p.kc, row0, af, ch >= 0 && ch < nkc);
        __syncwarp();
        if (lane == 0) {
          __threadfence_block();
          *reinterpret_cast<volatile int*>(&hdr->a_ticket) = (run >> 1) + 1;
        }
      }
    }
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->empty[stage]), phase ^ 1u, ctl,
                                                              ST_TIMEOUT_PRODUCER));
    if (!ok) break;
    const uint32_t sb = stage0 + static_cast<uint32_t>(stage) * p.stage_bytes;
    const uint32_t full = baddr(&hdr->full[stage]);
    mbar_arrive_expect_tx_pred(full, (kKeepA ? 0u : a_bytes) + static_cast<uint32_t>(nseg) * seg_bytes,
                               lane == 0);
    // lanes 0..nseg-1: one B segment each; lane 8: the 128-row A box
    tma_load_2d_pred(sb + b_off + static_cast<uint32_t>(lane & 7) * seg_bytes, &p.tm_b, my_col,
                     kci * p.kc, full, lane < nseg);
    if (!kKeepA) tma_load_2d_pred(sb, &p.tm_a, kci * p.kc, row0, full, lane == 8);
    armed |= 1u << stage;
    armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
    stage += P;
    if (stage >= p.stages) {
      stage -= p.stages;
      phase ^= 1u;
    }
  }
  if (lane == 0) {
#pragma unroll 1
    for (int s = 0; s < p.stages; ++s)
      if (armed & (1u << s)) sd_drain_wait(baddr(&hdr->full[s]), (armed_parity >> s) & 1u, ctl);
  }
  __syncwarp();
}

// MMA warp: every lane waits, lane 0 issues (predicated, no divergence).
// kKeepA: A comes from the run's resident buffer; the buffer is released
// (a_empty) after the run's last unit.
template <int kKS, bool kKeepA>
__device__ __forceinline__ void sd_mma(const SddmmKernelParams& p, SdSmemHeader* hdr, uint32_t stage0,
                                      uint32_t abuf0, uint32_t tmem_base, int u_begin, int u_end,
                                      const WaitCtl& ctl, int lane) {
  const uint32_t is0 = lane == 0 ? 1u : 0u;
  const int nkc = p.nkc;
  // A: K-major 128 rows of kc*2 bytes (128B swizzle for kc = 64, 64B for 32),
  //    SBO = 8 rows; a 16-column k-step is 32 bytes.
  // B: MN-major 64B swizzle, LBO = one 32-column segment (kc rows x 64 B),
  //    SBO = 8 k-rows of 64 B; a 16-row k-step is 1024 bytes.
  const uint32_t a_sbo = (p.a_swizzle_mode == 2) ? 1024u : 512u;
  const uint64_t adesc0 = smem_desc(kKeepA ? abuf0 : stage0, 16u, a_sbo, static_cast<uint32_t>(p.a_swizzle_mode));
  const uint64_t bdesc0 = smem_desc(stage0 + (kKeepA ? 0u : static_cast<uint32_t>(p.a_bytes)),
                                    static_cast<uint32_t>(p.seg_bytes), 512u, 4u);
  const uint32_t a16 = static_cast<uint32_t>(p.a_bytes) >> 4;  // one k-chunk of the A tile
  const uint32_t abuf16 = a16 * static_cast<uint32_t>(p.nkc);  // one A buffer
  uint32_t abuf = 0;
  const uint32_t idesc = idesc_bf16_f32(128, 32 * p.nseg_max, /*a K-major*/ 0, /*b MN-major*/ 1);
  const uint32_t stage16 = static_cast<uint32_t>(p.stage_bytes) >> 4;
  const uint32_t full0 = baddr(&hdr->full[0]);
  const uint32_t empty0 = baddr(&hdr->empty[0]);
  const uint32_t acc_cols = 32u * static_cast<uint32_t>(p.nseg_max);  // TMEM columns per buffer
  int stage = 0;
  uint32_t phase = 0, soff = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    if (!__all_sync(0xffffffffu,
                    mbar_wait_bounded(baddr(&hdr->acc_empty[acc]), acc_phase ^ 1u, ctl, ST_TIMEOUT_MMA)))
      break;
    int32_t run = 0, last = 0;
    if (kKeepA) {
      run = __ldg(&p.rs_units[u].pad[0]);
      last = __ldg(&p.rs_units[u].pad[1]);
      if (run & 1) {
        abuf = static_cast<uint32_t>(run >> 1) & 1u;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->a_full[abuf]),
                                                        static_cast<uint32_t>(run >> 2) & 1u, ctl,
                                                        ST_TIMEOUT_MMA)))
          break;
      }
    }
    tc_fence_after();
    const uint32_t d = tmem_base + static_cast<uint32_t>(acc) * acc_cols;
    bool ok = true;
#pragma unroll 1
    for (int kci = 0; kci < nkc; ++kci) {
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(full0 + stage * 8, phase, ctl, ST_TIMEOUT_MMA))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t ad = kKeepA ? adesc0 + abuf * abuf16 + static_cast<uint32_t>(kci) * a16 : adesc0 + soff;
#pragma unroll
      for (int k = 0; k < kKS; ++k)
        mma_bf16_pred(d, ad + k * 2u, bdesc0 + soff + k * 64u, idesc, (kci | k) != 0, is0);
      mma_commit_pred(empty0 + stage * 8, is0);
      soff += stage16;
      if (++stage == p.stages) {
        stage = 0;
        soff = 0;
        phase ^= 1u;
      }
    }
    if (!ok) break;
    mma_commit_pred(baddr(&hdr->acc_full[acc]), is0);
    if (kKeepA && last) mma_commit_pred(baddr(&hdr->a_empty[abuf]), is0);
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1u;
  }
  if (lane == 0) {
    mma_commit(baddr(&hdr->drain));
    sd_drain_wait(baddr(&hdr->drain), 0, ctl);
  }
  __syncwarp();
}

// Epilogue warp of slab q = warp & 3, segments of parity h = (warp - 4) >> 2:
// thread r holds output row row0 + 32q + r; for each segment the mask holds,
// one TMEM load gives the row's 32 columns, written as 64 contiguous bytes of
// the output block (the warp writes 32 rows of it).  The next tile's TMEM
// load is in flight while the current tile is converted and stored.
__device__ __forceinline__ void sd_store_tile(const SddmmKernelParams& p, int64_t e, const uint32_t (&v)[32]) {
  uint4* dst = reinterpret_cast<uint4*>(p.out_vals + e);
  if (p.mask_vals) {
    const uint4* mk = reinterpret_cast<const uint4*>(p.mask_vals + e);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 m4 = __ldg(mk + i);
      const uint32_t mw[4] = {m4.x, m4.y, m4.z, m4.w};
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float m0 = __uint_as_float(mw[h] << 16), m1 = __uint_as_float(mw[h] & 0xFFFF0000u);
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(m0 * __uint_as_float(v[8 * i + 2 * h]),
                                                        m1 * __uint_as_float(v[8 * i + 2 * h + 1]));
        w[h] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(v[8 * i + 2 * h]),
                                                        __uint_as_float(v[8 * i + 2 * h + 1]));
        w[h] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

__device__ __forceinline__ void sd_epilogue(const SddmmKernelParams& p, SdSmemHeader* hdr,
                                           uint32_t tmem_base, int u_begin, int u_end,
                                           const WaitCtl& ctl, int warp, int lane) {
  const int q = warp & 3;
  const int half = (warp - kSdEpi0) >> 2;
  const int64_t blk_elems = static_cast<int64_t>(p.R) * p.C;
  const uint32_t acc_cols = 32u * static_cast<uint32_t>(p.nseg_max);
  const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
  int acc = 0;
  uint32_t acc_phase = 0;
  // lane s < 8 holds (seg_col[s], blk[q][s]) of the unit
  auto load = [&](int u, int32_t* col, int32_t* blk, int32_t* row0) {
    const SddmmRsUnit* un = p.rs_units + u;
    *row0 = __ldg(&un->row0);
    *col = lane < kSddmmRsMaxSeg ? __ldg(&un->seg_col[lane]) : -1;
    *blk = lane < kSddmmRsMaxSeg ? __ldg(&un->blk[q][lane]) : -1;
  };
  int32_t n_col = -1, n_blk = -1, n_row0 = 0;
  if (u_begin < u_end) load(u_begin, &n_col, &n_blk, &n_row0);
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    const int32_t col = n_col, blk = n_blk, row0 = n_row0;
    if (u + 1 < u_end) load(u + 1, &n_col, &n_blk, &n_row0);
    if (!mbar_wait_bounded(baddr(&hdr->acc_full[acc]), acc_phase, ctl, ST_TIMEOUT_EPILOGUE)) break;
    tc_fence_after();
    const int64_t row = static_cast<int64_t>(row0) + 32 * q;  // first row of the slab
    const int64_t rib = row % p.R;                             // its row inside the block
    const uint32_t acc_base = lane_base + static_cast<uint32_t>(acc) * acc_cols;
    // this warp's tiles: segments of parity `half` that the mask holds
    uint32_t m = __ballot_sync(0xffffffffu, lane < kSddmmRsMaxSeg && (lane & 1) == half && blk >= 0);
    // output element of (segment s, this thread's row)
    auto elem = [&](int s) {
      const int32_t b = __shfl_sync(0xffffffffu, blk, s);
      const int32_t c = __shfl_sync(0xffffffffu, col, s);
      return static_cast<int64_t>(b) * blk_elems + (rib + lane) * p.C + (c % p.C);
    };
    uint32_t va[32], vb[32];
    int sa = -1, sb = -1;
    if (m) {
      sa = __ffs(m) - 1;
      m &= m - 1;
      tmem_ld_32x32b_x32(acc_base + static_cast<uint32_t>(sa * 32), va);
    }
#pragma unroll 1
    while (sa >= 0) {
      tmem_ld_wait_regs(va);
      sb = -1;
      if (m) {
        sb = __ffs(m) - 1;
        m &= m - 1;
        tmem_ld_32x32b_x32(acc_base + static_cast<uint32_t>(sb * 32), vb);
      }
      sd_store_tile(p, elem(sa), va);
      if (sb < 0) break;
      tmem_ld_wait_regs(vb);
      sa = -1;
      if (m) {
        sa = __ffs(m) - 1;
        m &= m - 1;
        tmem_ld_32x32b_x32(acc_base + static_cast<uint32_t>(sa * 32), va);
      }
      sd_store_tile(p, elem(sb), vb);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(baddr(&hdr->acc_empty[acc]));
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1u;
  }
}

__global__ void __launch_bounds__(kSdThreads, 1) sddmm_rowstack_tcgen05(const __grid_constant__ SddmmKernelParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  SdSmemHeader* hdr = reinterpret_cast<SdSmemHeader*>(gbase);
  // resident-A buffers (keep_a) sit between the header and the stage ring
  const uint32_t abuf0 = base + 1024u;
  const uint32_t stage0 = abuf0 + (p.keep_a ? 2u * static_cast<uint32_t>(p.a_bytes) * static_cast<uint32_t>(p.nkc) : 0u);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int u_begin = p.cta_begin[blockIdx.x];
  const int u_end = p.cta_begin[blockIdx.x + 1];

  if (threadIdx.x == 32) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(baddr(&hdr->full[s]), 1);
      mbar_init(baddr(&hdr->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(baddr(&hdr->acc_full[a]), 1);
      mbar_init(baddr(&hdr->acc_empty[a]), kSdEpiWarps);
      mbar_init(baddr(&hdr->a_full[a]), 1);
      mbar_init(baddr(&hdr->a_empty[a]), 1);
    }
    mbar_init(baddr(&hdr->drain), 1);
    hdr->abort_flag = 0;
    hdr->a_ticket = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
  }
  if (warp == kSdMmaWarp) {
    tmem_alloc(smem_u32(&hdr->tmem_base), static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = hdr->tmem_base;
  const WaitCtl ctl{&hdr->abort_flag, p.status, p.timeout_ns};

  if (warp == kSdMmaWarp) {
    if (p.keep_a) {
      if (p.kc == 64) sd_mma<4, true>(p, hdr, stage0, abuf0, tmem_base, u_begin, u_end, ctl, lane);
      else sd_mma<2, true>(p, hdr, stage0, abuf0, tmem_base, u_begin, u_end, ctl, lane);
    } else {
      if (p.kc == 64) sd_mma<4, false>(p, hdr, stage0, abuf0, tmem_base, u_begin, u_end, ctl, lane);
      else sd_mma<2, false>(p, hdr, stage0, abuf0, tmem_base, u_begin, u_end, ctl, lane);
    }
  } else if (warp < kSdEpi0) {
    if (warp - kSdProd0 < p.nprod) {
      if (p.keep_a) sd_producer<true>(p, hdr, stage0, abuf0, u_begin, u_end, ctl, warp - kSdProd0, lane);
      else sd_producer<false>(p, hdr, stage0, abuf0, u_begin, u_end, ctl, warp - kSdProd0, lane);
    }
  } else {
    sd_epilogue(p, hdr, tmem_base, u_begin, u_end, ctl, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kSdMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
  // Resident A tiles still in flight (a role gave up early): wait for the
  // latest load of each buffer.  Tiles were issued in run order, so the last
  // two runs issued hold the buffers' latest phases (a producer's own record
  // of a buffer can be a phase behind when another warp reloaded it).
  if (p.keep_a && threadIdx.x == kSdProd0 * 32) {
    const int issued = *reinterpret_cast<volatile int*>(&hdr->a_ticket);
    for (int r = issued - 2; r < issued; ++r)
      if (r >= 0) sd_drain_wait(baddr(&hdr->a_full[r & 1]), static_cast<uint32_t>(r >> 1) & 1u, ctl);
  }
}

}  // namespace

int sddmm_rowstack_max_stages() { return kSdMaxStages; }
int sddmm_rowstack_max_producers() { return kSdMaxProducers; }

bsp_status launch_sddmm_rowstack(const bsp_sddmm_plan* p, const bsp_bsr_desc* mask, const void* A,
                                 int64_t lda, const void* B, int64_t ldb, void* out,
                                 cudaStream_t stream) {
  if (p->n_units == 0) return BSP_OK;
  bsp_device* dev = p->dev;
  if (reinterpret_cast<uintptr_t>(A) % 16 || (lda * 2) % 16 || reinterpret_cast<uintptr_t>(B) % 16 ||
      (ldb * 2) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "A and B must be 16-byte aligned with 16-byte row pitch");
  if (mask->values && reinterpret_cast<uintptr_t>(mask->values) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "mask values must be 16-byte aligned");
  SddmmKernelParams kp;
  memset(&kp, 0, sizeof(kp));
  const CUtensorMapSwizzle a_swz = p->kc == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  bsp_status st = encode_2d(dev, &kp.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, p->K, p->M, lda, p->kc,
                            128, a_swz);
  if (st != BSP_OK) return st;
  st = encode_2d(dev, &kp.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, p->N, p->K, ldb, 32, p->kc,
                 CU_TENSOR_MAP_SWIZZLE_64B);
  if (st != BSP_OK) return st;
  kp.rs_units = p->d_rs_units;
  kp.cta_begin = p->d_cta_begin;
  kp.mask_vals = static_cast<const uint16_t*>(mask->values);
  kp.out_vals = static_cast<uint16_t*>(out);
  kp.status = dev->d_status;
  kp.timeout_ns = p->timeout_ns;
  kp.R = p->R;
  kp.C = p->C;
  kp.Rs = 32;
  kp.kc = p->kc;
  kp.nkc = static_cast<int32_t>(p->K / p->kc);
  kp.stages = p->stages;
  kp.stage_bytes = p->stage_bytes;
  kp.a_bytes = 128 * p->kc * 2;
  kp.a_swizzle_mode = p->kc == 64 ? 2 : 4;
  kp.tmem_cols = p->tmem_cols;
  kp.M = static_cast<int32_t>(p->M);
  kp.nseg_max = p->nseg_max;
  kp.nprod = p->nprod;
  kp.seg_bytes = p->kc * 64;
  kp.keep_a = p->keep_a;
  cudaError_t e = cudaFuncSetAttribute(sddmm_rowstack_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       p->smem_bytes);
  if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(sddmm rowstack)");
  sddmm_rowstack_tcgen05<<<p->grid, kSdThreads, p->smem_bytes, stream>>>(kp);
  return cuda_check(cudaGetLastError(), "sddmm rowstack kernel launch");
}

}  // namespace bsp
