// BSR x BSR -> BSR SpGEMM on sm_100a tensor cores:
//   C(i, j) = sum_k A(i, k) * B(k, j)   for every block (i, j) of C's pattern.
//
// Reference: bsr_matrix<T>::spgemm (sparse_common/bsr_matrix.hpp:741-810), a
// CPU loop over A's blocks and the matching rows of B with fp32 block
// accumulators; the reference has no device version.
//
// Mapping (planner.cpp, plan_spgemm_host): a work unit stacks four 32-row
// "entries" (slabs of output block-rows) into MMA M = 128 and gathers up to
// eight 32-column "segments" of output block-columns into MMA N = 256.  Its
// steps walk the shared block index k; a step is one TMA box per entry (the
// slab of A(i_e, k), K-major) and one per segment (32 columns of B(k, j_s),
// MN-major, 64B swizzle), absent blocks being boxes placed wholly outside the
// tensor, which TMA fills with zeros.  K = Ca runs in kc-wide sub-steps
// (kc/16 MMAs each), `sps` sub-steps per pipeline stage.  The fp32
// accumulator (128 lanes x 32*nseg_max columns) sits in TMEM, double-buffered;
// the epilogue writes each (entry, segment) tile whose output block exists,
// rounded once to bf16, into C's block layout.  Every output block belongs to
// exactly one unit, so there are no atomics and no second pass.
//
// Warp roles (256 threads, one persistent CTA per SM):
//   warp 0      TMEM allocator + MMA issuer (converged warp, lane 0 issues)
//   warps 1..3  TMA producers: producer w issues the CTA's stages w, w + P, ...;
//               one predicated instruction issues the entry boxes (lanes 0..7,
//               two sub-steps) and another the segment boxes (lanes 8..23)
//   warps 4..7  epilogue (TMEM lane quarter q = entry q)
// Every wait is bounded (bsp_ptx.cuh).
#include <cuda_bf16.h>

#include <cstddef>

#include "bsp_internal.h"
#include "bsp_ptx.cuh"

namespace bsp {
using namespace dev;

namespace {

constexpr int kSgMmaWarp = 0;
constexpr int kSgProd0 = 1;
constexpr int kSgMaxProducers = 3;
constexpr int kSgEpi0 = 4;
constexpr int kSgThreads = 8 * 32;
constexpr int kSgMaxStages = 24;
constexpr int kSgMaxSps = 4;
constexpr int kStepWords = sizeof(SpgemmStep) / 4;

struct SgSmemHeader {
  uint64_t full[kSgMaxStages];
  uint64_t empty[kSgMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(SgSmemHeader) <= 1024, "header must fit its 1 KiB slot");

__device__ __forceinline__ uint32_t baddr(const uint64_t* b) { return smem_u32(b); }

__device__ __noinline__ bool sg_drain_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl) {
  int zero = 0;
  WaitCtl c2{&zero, ctl.status, ctl.timeout_ns};
  return mbar_wait_bounded(bar, parity, c2, ST_TIMEOUT_DRAIN);
}

// Lane roles inside one issue round (two sub-steps): lanes 0..7 entry boxes
// (sub-step lane>>2, box lane&3), lanes 8..23 segment boxes (sub-step
// (lane-8)>>3, box (lane-8)&7).
__device__ __forceinline__ int lane_sub(int lane) { return lane < 8 ? (lane >> 2) : ((lane - 8) >> 3); }
__device__ __forceinline__ int lane_idx(int lane) { return lane < 8 ? (lane & 3) : ((lane - 8) & 7); }

// Producer warp pw of P: the CTA's stage sequence is unit-major (unit u has
// ceil(n_steps * nkc / sps) stages); this warp issues every P-th of them.
// The step words of the next owned stage are fetched while the current one
// waits for its slot and issues, so their latency stays off the critical path.
struct SgCursor {
  int u;            // unit (u_end: done)
  int ls;           // stage inside the unit
  int64_t seq;      // CTA stages before the unit
  int ns, total_sub, step_begin, nseg;
};

__device__ __forceinline__ void sg_load_unit(const SpgemmKernelParams& p, SgCursor* c, int my_idx) {
  const SpgemmUnit* un = p.units + c->u;
  const int n_steps = __ldg(&un->n_steps);
  c->step_begin = __ldg(&un->step_begin);
  c->nseg = __ldg(&un->nseg);
  c->total_sub = n_steps * p.nkc;
  c->ns = (c->total_sub + p.sps - 1) / p.sps;
}

// Move to the next stage this producer owns (P stages further on).
__device__ __forceinline__ void sg_advance(const SpgemmKernelParams& p, SgCursor* c, int u_end, int P,
                                           int my_idx) {
  c->ls += P;
  while (c->ls >= c->ns) {
    c->ls -= c->ns;
    c->seq += c->ns;
    if (++c->u >= u_end) return;
    sg_load_unit(p, c, my_idx);
  }
}

__device__ __forceinline__ void sg_producer(const SpgemmKernelParams& p, SgSmemHeader* hdr,
                                           uint32_t stage0, int u_begin, int u_end,
                                           const WaitCtl& ctl, int pw, int lane) {
  const int P = p.nprod;
  const int sps = p.sps, kc = p.kc;
  const uint32_t a_slot = static_cast<uint32_t>(p.a_slot);
  const uint32_t seg_bytes = static_cast<uint32_t>(p.seg_bytes);
  const uint32_t a_all = kSpgemmEnt * a_slot;
  const int32_t* step_words = reinterpret_cast<const int32_t*>(p.steps);
  const bool is_a = lane < 8;
  const int my_sub = lane_sub(lane);
  const int my_idx = lane_idx(lane);
  const int my_word = is_a ? my_idx : kSpgemmEnt + my_idx;
  const int my_meta = is_a ? offsetof(SpgemmStep, a_meta) + my_idx : offsetof(SpgemmStep, b_meta) + my_idx;
  uint32_t armed = 0, armed_parity = 0;

  // this lane's box of a stage (up to two issue rounds of two sub-steps):
  // its coordinate word and its meta byte
  struct Words {
    int32_t w[kSgMaxSps / 2];
    uint32_t meta[kSgMaxSps / 2];
    int kci[kSgMaxSps / 2];
    int n_sub;
  };
  auto fetch = [&](const SgCursor& c, Words* W) {
    W->n_sub = min(sps, c.total_sub - c.ls * sps);
#pragma unroll
    for (int r = 0; r < kSgMaxSps / 2; ++r) {
      const int sub = 2 * r + my_sub;
      const bool in = lane < 24 && sub < W->n_sub;
      const int fs = c.ls * sps + sub;
      const int step = fs / p.nkc;
      W->kci[r] = fs - step * p.nkc;
      const int64_t rec = static_cast<int64_t>(c.step_begin + step) * kStepWords;
      W->w[r] = in ? __ldg(step_words + rec + my_word) : 0;
      W->meta[r] = in ? __ldg(reinterpret_cast<const uint8_t*>(step_words + rec) + my_meta) : 0u;
    }
  };

  SgCursor cur{u_begin, 0, 0, 0, 0, 0, 0};
  if (cur.u < u_end) {
    sg_load_unit(p, &cur, my_idx);
    // first owned stage: pw (stages are numbered from 0 across the CTA's units)
    cur.ls = pw - P;
    sg_advance(p, &cur, u_end, P, my_idx);
  }
  Words wc;
  if (cur.u < u_end) fetch(cur, &wc);
#pragma unroll 1
  while (cur.u < u_end) {
    SgCursor nxt = cur;
    sg_advance(p, &nxt, u_end, P, my_idx);
    Words wn;
    if (nxt.u < u_end) fetch(nxt, &wn);
    const int64_t gs = cur.seq + cur.ls;
    const int slot = static_cast<int>(gs % p.stages);
    const uint32_t phase = static_cast<uint32_t>((gs / p.stages) & 1);
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->empty[slot]), phase ^ 1u, ctl,
                                                              ST_TIMEOUT_PRODUCER));
    if (!ok) break;
    const uint32_t sb = stage0 + static_cast<uint32_t>(slot) * p.stage_bytes;
    const uint32_t full = baddr(&hdr->full[slot]);
    mbar_arrive_expect_tx_pred(full, static_cast<uint32_t>(wc.n_sub) * (a_all + cur.nseg * seg_bytes),
                               lane == 0);
#pragma unroll
    for (int r = 0; r < kSgMaxSps / 2; ++r) {
      if (2 * r >= wc.n_sub) break;  // warp-uniform
      const uint32_t m = wc.meta[r];
      const bool valid = (m & kSpgemmBoxValid) != 0;
      const uint32_t first = m & 7u, lg = (m >> 3) & 3u;
      const uint32_t sub_base = sb + static_cast<uint32_t>(2 * r + my_sub) * p.sub_bytes;
      // entries: rows of A (slabs of blocks) at k-offset kci*kc, 32 << lg rows
      tma_load_2d_pred(sub_base + first * a_slot, &p.tm_a[min(lg, 2u)], wc.kci[r] * kc,
                       wc.w[r], full, valid && is_a);
      // segments: slice t of 1 << lg consecutive blocks of B at k-offset kci*kc
      tma_load_3d_pred(sub_base + a_all + first * seg_bytes, &p.tm_b[lg], static_cast<int32_t>((m >> 5) & 3u) * 32,
                       wc.kci[r] * kc, wc.w[r], full, valid && !is_a);
    }
    armed |= 1u << slot;
    armed_parity = (armed_parity & ~(1u << slot)) | (phase << slot);
    cur = nxt;
    wc = wn;
  }
  if (lane == 0) {
#pragma unroll 1
    for (int s = 0; s < p.stages; ++s)
      if (armed & (1u << s)) sg_drain_wait(baddr(&hdr->full[s]), (armed_parity >> s) & 1u, ctl);
  }
  __syncwarp();
}

// MMA warp: every lane waits, lane 0 issues (predicated, no divergence).
template <int kKS>
__device__ __forceinline__ void sg_mma(const SpgemmKernelParams& p, SgSmemHeader* hdr, uint32_t stage0,
                                      uint32_t tmem_base, int u_begin, int u_end, const WaitCtl& ctl,
                                      int lane) {
  const uint32_t is0 = lane == 0 ? 1u : 0u;
  const int nkc = p.nkc, sps = p.sps;
  // A: K-major, 128 rows (4 entry slots of 32) of kc*2 bytes, SBO = 8 rows;
  //    a 16-column k-step is 32 bytes.
  // B: MN-major 64B swizzle, LBO = one segment (kc rows x 64 B), SBO = 8 k-rows
  //    of 64 B; a 16-row k-step is 1024 bytes.
  const uint32_t a_sbo = (p.a_swizzle_mode == 2) ? 1024u : 512u;
  const uint64_t adesc0 = smem_desc(stage0, 16u, a_sbo, static_cast<uint32_t>(p.a_swizzle_mode));
  const uint64_t bdesc0 = smem_desc(stage0 + static_cast<uint32_t>(kSpgemmEnt * p.a_slot),
                                    static_cast<uint32_t>(p.seg_bytes), 512u, 4u);
  const uint32_t idesc = idesc_bf16_f32(128, 32 * p.nseg_max, /*a K-major*/ 0, /*b MN-major*/ 1);
  const uint32_t stage16 = static_cast<uint32_t>(p.stage_bytes) >> 4;
  const uint32_t sub16 = static_cast<uint32_t>(p.sub_bytes) >> 4;
  const uint32_t full0 = baddr(&hdr->full[0]);
  const uint32_t empty0 = baddr(&hdr->empty[0]);
  const uint32_t acc_cols = 32u * static_cast<uint32_t>(p.nseg_max);
  int stage = 0;
  uint32_t phase = 0, soff = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  bool ok = true;
#pragma unroll 1
  for (int u = u_begin; u < u_end && ok; ++u) {
    const int total_sub = __ldg(&p.units[u].n_steps) * nkc;
    const int ns = (total_sub + sps - 1) / sps;
    if (!__all_sync(0xffffffffu,
                    mbar_wait_bounded(baddr(&hdr->acc_empty[acc]), acc_phase ^ 1u, ctl, ST_TIMEOUT_MMA)))
      break;
    tc_fence_after();
    const uint32_t d = tmem_base + static_cast<uint32_t>(acc) * acc_cols;
#pragma unroll 1
    for (int ls = 0; ls < ns; ++ls) {
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(full0 + stage * 8, phase, ctl, ST_TIMEOUT_MMA))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int n_sub = min(sps, total_sub - ls * sps);
#pragma unroll 1
      for (int sub = 0; sub < n_sub; ++sub) {
        const uint32_t o = soff + static_cast<uint32_t>(sub) * sub16;
#pragma unroll
        for (int k = 0; k < kKS; ++k)
          mma_bf16_pred(d, adesc0 + o + k * 2u, bdesc0 + o + k * 64u, idesc, (ls | sub | k) != 0, is0);
      }
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
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1u;
  }
  if (lane == 0) {
    mma_commit(baddr(&hdr->drain));
    sg_drain_wait(baddr(&hdr->drain), 0, ctl);
  }
  __syncwarp();
}

// Epilogue warp of entry q: thread r holds row ent_r + r of the entry's output
// block-row; each segment with an output block gives one TMEM load of 32
// columns, written as 64 contiguous bytes (the warp writes 32 rows).
__device__ __forceinline__ void sg_epilogue(const SpgemmKernelParams& p, SgSmemHeader* hdr,
                                           uint32_t tmem_base, int u_begin, int u_end,
                                           const WaitCtl& ctl, int warp, int lane) {
  const int q = warp & 3;
  const int64_t blk_elems = static_cast<int64_t>(p.Ra) * p.Cb;
  const uint32_t acc_cols = 32u * static_cast<uint32_t>(p.nseg_max);
  int acc = 0;
  uint32_t acc_phase = 0;
  // lane s < 8 holds (out_blk[q][s], seg_x[s]); every lane holds ent_r[q]
  auto load = [&](int u, int32_t* blk, int32_t* sx, int32_t* er) {
    const SpgemmUnit* un = p.units + u;
    *blk = lane < kSpgemmMaxSeg ? __ldg(&un->out_blk[q][lane]) : -1;
    *sx = lane < kSpgemmMaxSeg ? __ldg(&un->seg_x[lane]) : 0;
    *er = __ldg(&un->ent_r[q]);
  };
  int32_t n_blk = -1, n_sx = 0, n_er = 0;
  if (u_begin < u_end) load(u_begin, &n_blk, &n_sx, &n_er);
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    const int32_t blk = n_blk, sx = n_sx, er = n_er;
    if (u + 1 < u_end) load(u + 1, &n_blk, &n_sx, &n_er);
    if (!mbar_wait_bounded(baddr(&hdr->acc_full[acc]), acc_phase, ctl, ST_TIMEOUT_EPILOGUE)) break;
    tc_fence_after();
#pragma unroll 1
    for (int s = 0; s < kSpgemmMaxSeg; ++s) {
      const int32_t b = __shfl_sync(0xffffffffu, blk, s);
      if (b < 0) continue;  // warp-uniform
      const int32_t x = __shfl_sync(0xffffffffu, sx, s);
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(acc) * acc_cols + static_cast<uint32_t>(s * 32),
                         v);
      tmem_ld_wait();
      const int64_t e = static_cast<int64_t>(b) * blk_elems + static_cast<int64_t>(er + lane) * p.Cb + x;
      uint4* dst = reinterpret_cast<uint4*>(p.out_vals + e);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t wv[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(v[8 * i + 2 * h]),
                                                          __uint_as_float(v[8 * i + 2 * h + 1]));
          wv[h] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        dst[i] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(baddr(&hdr->acc_empty[acc]));
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1u;
  }
}

__global__ void __launch_bounds__(kSgThreads, 1) spgemm_tcgen05(const __grid_constant__ SpgemmKernelParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  SgSmemHeader* hdr = reinterpret_cast<SgSmemHeader*>(smem_raw + (base - raw));
  const uint32_t stage0 = base + 1024u;
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
      mbar_init(baddr(&hdr->acc_empty[a]), 4);
    }
    mbar_init(baddr(&hdr->drain), 1);
    hdr->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_a[0]);
    tma_prefetch_desc(&p.tm_b[0]);
  }
  if (warp == kSgMmaWarp) {
    tmem_alloc(smem_u32(&hdr->tmem_base), static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = hdr->tmem_base;
  const WaitCtl ctl{&hdr->abort_flag, p.status, p.timeout_ns};

  if (warp == kSgMmaWarp) {
    if (p.kc == 64) sg_mma<4>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
    else sg_mma<2>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
  } else if (warp < kSgEpi0) {
    if (warp - kSgProd0 < p.nprod) sg_producer(p, hdr, stage0, u_begin, u_end, ctl, warp - kSgProd0, lane);
  } else {
    sg_epilogue(p, hdr, tmem_base, u_begin, u_end, ctl, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kSgMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
}

}  // namespace

int spgemm_max_stages() { return kSgMaxStages; }
int spgemm_max_producers() { return kSgMaxProducers; }

bsp_status launch_spgemm(const bsp_spgemm_plan* p, const void* a_vals, const void* b_vals, void* out_vals,
                         cudaStream_t stream) {
  if (p->n_units == 0) return BSP_OK;
  if (p->sps < 1 || p->sps > kSgMaxSps || p->stages < 2 || p->stages > kSgMaxStages ||
      p->stages % p->nprod || p->nprod < 1 || p->nprod > kSgMaxProducers)
    return set_error(BSP_ERR_STATE, "inconsistent SpGEMM plan");
  bsp_device* dev = p->dev;
  if (reinterpret_cast<uintptr_t>(a_vals) % 16 || reinterpret_cast<uintptr_t>(b_vals) % 16 ||
      reinterpret_cast<uintptr_t>(out_vals) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "A, B and C values must be 16-byte aligned");
  SpgemmKernelParams kp;
  memset(&kp, 0, sizeof(kp));
  const CUtensorMapSwizzle a_swz = p->kc == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  // one map per box size; sizes larger than the tensor are never used
  for (int l = 0; l <= p->la_log2; ++l) {
    bsp_status st = encode_2d(dev, &kp.tm_a[l], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a_vals, p->Ca,
                              static_cast<uint64_t>(p->nnzb_a) * p->Ra, p->Ca, p->kc, 32u << l, a_swz);
    if (st != BSP_OK) return st;
  }
  for (int l = 0; l <= p->lb_log2; ++l) {
    const uint64_t dims[3] = {static_cast<uint64_t>(p->Cb), static_cast<uint64_t>(p->Ca),
                              static_cast<uint64_t>(p->nnzb_b)};
    const uint64_t strides[2] = {static_cast<uint64_t>(p->Cb) * 2, static_cast<uint64_t>(p->Ca) * p->Cb * 2};
    const uint32_t box[3] = {32, static_cast<uint32_t>(p->kc), 1u << l};
    bsp_status st = encode_nd(dev, &kp.tm_b[l], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, b_vals, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_64B);
    if (st != BSP_OK) return st;
  }
  kp.units = p->d_units;
  kp.steps = p->d_steps;
  kp.cta_begin = p->d_cta_begin;
  kp.out_vals = static_cast<uint16_t*>(out_vals);
  kp.status = dev->d_status;
  kp.timeout_ns = p->timeout_ns;
  kp.Ra = p->Ra;
  kp.Cb = p->Cb;
  kp.kc = p->kc;
  kp.nkc = p->nkc;
  kp.sps = p->sps;
  kp.stages = p->stages;
  kp.stage_bytes = p->stage_bytes;
  kp.sub_bytes = p->sub_bytes;
  kp.a_slot = 32 * p->kc * 2;
  kp.seg_bytes = p->kc * 64;
  kp.a_swizzle_mode = p->kc == 64 ? 2 : 4;
  kp.tmem_cols = p->tmem_cols;
  kp.nseg_max = p->nseg_max;
  kp.nprod = p->nprod;
  cudaError_t e = cudaFuncSetAttribute(spgemm_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       p->smem_bytes);
  if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(spgemm)");
  spgemm_tcgen05<<<p->grid, kSgThreads, p->smem_bytes, stream>>>(kp);
  return cuda_check(cudaGetLastError(), "spgemm kernel launch");
}

}  // namespace bsp
