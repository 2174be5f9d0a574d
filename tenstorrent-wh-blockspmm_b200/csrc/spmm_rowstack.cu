// BSR SpMM on sm_100a tensor cores, "row-stacked" form used by the DDA
// strategy:  C[M x N] = A_bsr[M x K] * B[K x N].
//
// The tensor pipe takes ~135 cycles per M=128 x K=16 MMA whatever N is (up to
// 256), so only N = 256 MMAs reach full rate.  This kernel therefore keeps the
// natural orientation and fills the MMA with block-sparse structure:
//   MMA M = 128 output rows = G = 128/Rs "entries" (an entry is an Rs-row slab
//           of one block-row) stacked on top of each other; at each step the
//           entries' blocks of the same block-column j are loaded side by side
//           (K-major operand, absent entries zero-filled), so ONE load of the
//           dense slice B[j*C : (j+1)*C, n0 : n0+256] serves every entry that
//           has a block in column j -- the B-slice sharing the reference's
//           chain of direct addressing gives (block_spmm/kernels/dataflow/
//           reader_in1_chain_of_direct_addressing.cpp:257-367), here inside
//           one CTA's shared memory;
//   MMA N = 256 dense columns (MN-major B operand, four 64-column 128B-swizzle
//           boxes from one 3-D TMA load), so every A block is reused across
//           256 columns (the store-and-forward reuse of in0); a B of at most
//           128 columns takes 128-column tiles (N = 128, two boxes) instead;
//   MMA K = C, in chunks of kc per pipeline stage, 16 per MMA.
// The fp32 accumulator (128 lanes = output rows x 256 columns) sits in TMEM,
// double-buffered; an epilogue thread owns one output row and writes 32
// consecutive columns per TMEM load with 16-byte vector stores.
//
// Warp roles (256 threads, one CTA per SM, persistent over its unit list):
//   warp 0      TMEM allocator + MMA issuer (one thread), alone on its SM
//               sub-partition apart from one mostly-idle epilogue warp
//   warps 1..3  TMA producers: warp w owns every nprod-th pipeline stage and
//               touches only the metadata of its own stages
//   warps 4..7  epilogue (TMEM lane quarters 0..3)
// Every wait is bounded (see bsp_ptx.cuh).
#include <cuda_bf16.h>

#include <type_traits>

#include "rowstack_common.cuh"

namespace bsp {
using namespace dev;
using namespace rs;

namespace {
// Producer warp pw (0-based among producers): issues the CTA's pipeline
// stages pw, pw + nprod, pw + 2*nprod, ... from the precomputed stage list.
// 32 of its stages are fetched at once (lane l holds the l-th, 64 bytes) and
// broadcast by shuffles, so the issuing lane never waits on global memory.
__device__ __forceinline__ void rs_producer(const SpmmKernelParams& p, RsSmemHeader* hdr,
                                           uint8_t* gbase, uint32_t base, uint32_t stage0,
                                           const WaitCtl& ctl, int pw, int lane) {
  const int P = p.nprod;
  const int k_begin = p.cta_stage_begin[blockIdx.x];
  const int n = p.cta_stage_begin[blockIdx.x + 1] - k_begin;
  const uint32_t a_slot = static_cast<uint32_t>(p.Rs * p.kc * 2);
  const uint32_t b_blk = static_cast<uint32_t>(p.kc * 128);  // one 64-column block
  const uint32_t nb = 2u * static_cast<uint32_t>(p.NT);        // 64-column blocks per tile (4 or 2)
  const uint32_t b_bytes = nb * b_blk;
  const uint32_t sub_bytes = static_cast<uint32_t>(p.sub_bytes);
  int stage = pw;
  uint32_t phase = 0;
  uint32_t armed = 0, armed_parity = 0;
  bool ok = true;
  const uint32_t is0 = lane == 0 ? 1u : 0u;
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
      ok = mbar_wait_bounded(baddr(&hdr->empty[stage]), phase ^ 1u, ctl, ST_TIMEOUT_PRODUCER);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (p.debug_drop_stage != 0 && blockIdx.x == 0 && k0 + j * P == p.debug_drop_stage - 1) {
        // testing: leave this stage unissued (nothing armed, nothing to drain);
        // the MMA warp's bounded wait on it runs out and the launch gives up
        stage += P;
        if (stage >= p.stages) {
          stage -= p.stages;
          phase ^= 1u;
        }
        continue;
      }
      const uint32_t sb = stage0 + static_cast<uint32_t>(stage) * p.stage_bytes;
      const uint32_t zero = (flags >> 8) & 0xFFu;
      if (zero) {
        // entry slots absent from their sub-step that still hold an older block
#pragma unroll 1
        for (uint32_t m = zero; m; m &= m - 1) {
          const int bit = __ffs(m) - 1;
          const uint32_t off = sb + (bit >> 2) * sub_bytes + b_bytes + (bit & 3) * a_slot;
          uint4* dst = reinterpret_cast<uint4*>(gbase + (off - base));
          for (uint32_t i = lane; i < a_slot / 16; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      // coordinates of this stage (all lanes take part in the shuffles)
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
      // Lane 0 issues; every lane runs the same (uniform) control flow and the
      // issuing instructions are predicated, so the warp never diverges here.
      if (lane == 0)
        hdr->info[stage] = flags & static_cast<uint32_t>(RS_FIRST | RS_LAST | RS_EMPTY | RS_TWO);
      __syncwarp();
      {
        const uint32_t full = baddr(&hdr->full[stage]);
        if (flags & RS_EMPTY) {
          mbar_arrive_pred(full, is0);
        } else {
          const uint32_t nsub = (flags & RS_TWO) ? 2u : 1u;
          const uint32_t np = (flags >> 16) & 0xFu;
          mbar_arrive_expect_tx_pred(full, nsub * b_bytes + np * a_slot, is0);
#pragma unroll
          for (uint32_t q = 0; q < 2; ++q) {
            if (q >= nsub) break;
            const uint32_t qb = sb + q * sub_bytes;
            const int ky = q ? ky1 : ky0;
            if (p.b3d) {
              tma_load_3d_pred(qb, &p.tm_b, 0, ky, bz, full, is0);
            } else {
#pragma unroll
              for (int h = 0; h < 4; ++h)
                if (h < static_cast<int>(nb)) tma_load_2d_pred(qb + h * b_blk, &p.tm_b, bz + h * 64, ky, full, is0);
            }
#pragma unroll
            for (int g = 0; g < kRsMaxG; ++g)
              if ((flags >> (4 * q + g)) & 1u)
                tma_load_2d_pred(qb + b_bytes + g * a_slot, &p.tm_a, ax, ay[4 * q + g], full, is0);
          }
        }
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
      }
      stage += P;
      if (stage >= p.stages) {
        stage -= p.stages;
        phase ^= 1u;
      }
    }
  }
  if (lane == 0) {
#pragma unroll 1
    for (int s = 0; s < p.stages; ++s)
      if (armed & (1u << s)) rs_drain_wait(baddr(&hdr->full[s]), (armed_parity >> s) & 1u, ctl);
  }
  __syncwarp();
}

// The whole MMA warp runs this loop without diverging: every lane waits on the
// barriers and executes the MMA and commit instructions predicated on lane 0.
// A lone lane looping while its 31 siblings sit at the CTA barrier, or an
// `if (lane == 0)` around the issue, costs hundreds of cycles per pipeline
// stage on sm_100.
template <int kKS>
__device__ __forceinline__ void rs_mma(const SpmmKernelParams& p, RsSmemHeader* hdr,
                                       uint32_t stage0, uint32_t tmem_base, int u_begin, int u_end,
                                       const WaitCtl& ctl, int lane) {
  int stage = 0;
  uint32_t phase = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  int units_left = u_end - u_begin;
  // A (stacked entries): K-major, rows of kc*2 bytes; B: MN-major 128B swizzle,
  // LBO = one 64-column block (kc rows x 128 B), SBO = 8 k-rows; a 16-row
  // k-step of B is 2048 bytes, a 16-column k-step of A is 32 bytes.
  // MMA N is the accumulator's width up to 256; a 512-column accumulator
  // takes two MMAs per k-step, the second on B's columns 256..511 (four
  // 64-column blocks further on in the slice)
  const uint32_t idesc = idesc_bf16_f32(128, min(p.acc_cols, 256), /*a K-major*/ 0, /*b MN-major*/ 1);
  const bool two_halves = p.acc_cols > 256;
  const uint32_t bhalf16 = static_cast<uint32_t>(4 * p.kc * 128) >> 4;
  const uint32_t b_bytes = static_cast<uint32_t>(2 * p.NT * p.kc * 128);
  const uint32_t a_sbo = (p.a_swizzle_mode == 2) ? 1024u : 512u;
  const uint64_t adesc0 = smem_desc(stage0 + b_bytes, 16u, a_sbo, static_cast<uint32_t>(p.a_swizzle_mode));
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
    // lanes agree on every wait's outcome, so a timeout leaves the loop warp-wide
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(full0 + stage * 8, phase, ctl, ST_TIMEOUT_MMA))) break;
    const uint32_t info = hdr->info[stage];
    const bool first = (info & RS_FIRST) != 0;
    if (first) {
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(baddr(&hdr->acc_empty[acc]), acc_phase ^ 1u, ctl, ST_TIMEOUT_MMA)))
        break;
      tc_fence_after();
      d0 = tmem_base + static_cast<uint32_t>(acc * p.acc_cols);
    }
    if (!(info & RS_EMPTY)) {
      const uint64_t ad = adesc0 + soff, bd = bdesc0 + soff;
#pragma unroll
      for (int k = 0; k < kKS; ++k)
        mma_bf16_pred(d0, ad + k * 2u, bd + k * 128u, idesc, (k > 0 || !first) ? 1u : 0u, is0);
      if (two_halves) {
#pragma unroll
        for (int k = 0; k < kKS; ++k)
          mma_bf16_pred(d0 + 256u, ad + k * 2u, bd + bhalf16 + k * 128u, idesc, (k > 0 || !first) ? 1u : 0u,
                        is0);
      }
      if (info & RS_TWO) {
#pragma unroll
        for (int k = 0; k < kKS; ++k)
          mma_bf16_pred(d0, ad + sub16 + k * 2u, bd + sub16 + k * 128u, idesc, 1u, is0);
      }
    }
    mma_commit_pred(empty0 + stage * 8, is0);
    if (info & RS_LAST) {
      mma_commit_pred(baddr(&hdr->acc_full[acc]), is0);
      if (p.n_acc != 1) acc ^= 1;
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
    mma_commit(baddr(&hdr->drain));
    rs_drain_wait(baddr(&hdr->drain), 0, ctl);
  }
  __syncwarp();
}

template <bool kF32>
__global__ void __launch_bounds__(kRsThreads, 1) spmm_rowstack_tcgen05(const __grid_constant__ SpmmKernelParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  RsSmemHeader* hdr = reinterpret_cast<RsSmemHeader*>(gbase);
  const uint32_t stage0 = base + 1024u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
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
      mbar_init(baddr(&hdr->acc_empty[a]), 4);
    }
    mbar_init(baddr(&hdr->drain), 1);
    mbar_init(baddr(&hdr->merge_bar), 4);  // the epilogue warps (split-K merge)
    hdr->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
  }
  if (warp == kRsMmaWarp) {
    tmem_alloc(smem_u32(&hdr->tmem_base), static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = hdr->tmem_base;
  const WaitCtl ctl{&hdr->abort_flag, p.status, p.timeout_ns};

  if (warp == kRsMmaWarp) {
    if (p.kc == 32) rs_mma<2>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
    else rs_mma<4>(p, hdr, stage0, tmem_base, u_begin, u_end, ctl, lane);
  } else if (warp < kRsEpi0) {
    if (warp - kRsProd0 < p.nprod) rs_producer(p, hdr, gbase, base, stage0, ctl, warp - kRsProd0, lane);
  } else {
    rs_epilogue<kF32>(p, hdr, tmem_base, u_begin, u_end, ctl, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kRsMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
}

}  // namespace

int rowstack_max_producers() { return kRsMaxProducers; }
int rowstack_max_stages() { return kRsMaxStages; }

bsp_status launch_spmm_rowstack(const bsp_spmm_plan* p, const bsp_bsr_desc* A, const void* B,
                                int64_t ldb, void* C, int64_t ldc, cudaStream_t stream,
                                void* const* peer_c, int n_peers) {
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && !peer_c))
    return set_error(BSP_ERR_INVALID_ARG, "n_peers must be 0..7 with a peer pointer each");
  for (int i = 0; i < n_peers; ++i)
    if (!peer_c[i] || reinterpret_cast<uintptr_t>(peer_c[i]) % 16)
      return set_error(BSP_ERR_INVALID_ARG, "peer C pointers must be non-null and 16-byte aligned");
  bsp_device* dev = p->dev;
  const bool f32 = p->c_type == BSP_F32;
  if (p->n_units == 0 || p->M == 0 || p->N == 0) return BSP_OK;
  if (reinterpret_cast<uintptr_t>(C) % 16 || (ldc * (f32 ? 4 : 2)) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "C must be 16-byte aligned with 16-byte row pitch");
  auto kern = f32 ? spmm_rowstack_tcgen05<true> : spmm_rowstack_tcgen05<false>;
  if (!p->attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p->smem_bytes);
    if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(spmm rowstack)");
    p->attr_set = true;
  }
  // Same operands as the previous call: reuse the encoded tensor maps.
  auto set_peers = [&](SpmmKernelParams& k) {
    k.n_peers = n_peers;
    for (int i = 0; i < kMaxPeers; ++i) k.peer_c[i] = i < n_peers ? peer_c[i] : nullptr;
  };
  if (p->kp_valid && p->kp_a == A->values && p->kp_b == B && p->kp_c == C && p->kp_ldb == ldb &&
      p->kp_ldc == ldc) {
    set_peers(p->kp);
    select_split_counters(p, p->kp);
    kern<<<p->grid, kRsThreads, p->smem_bytes, stream>>>(p->kp);
    return cuda_check(cudaGetLastError(), "spmm rowstack kernel launch");
  }
  SpmmKernelParams& kp = p->kp;
  p->kp_valid = false;
  memset(&kp, 0, sizeof(kp));
  bsp_status st;
  const CUtensorMapSwizzle a_swz = p->kc == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (p->nnzb > 0) {
    st = encode_2d(dev, &kp.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A->values, p->C,
                   static_cast<uint64_t>(p->nnzb) * p->R, p->C, p->kc, p->Rs, a_swz);
  } else {
    st = encode_2d(dev, &kp.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, p->N, p->K, ldb, p->kc,
                   p->Rs, a_swz);
  }
  if (st != BSP_OK) return st;
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
  kp.NT = p->NT;  // 128-column tiles per unit: 2 (MMA N = 256) or 1 (N = 128)
  kp.step_stride = p->step_stride;
  kp.c_f32 = f32;
  kp.stages = p->stages;
  kp.stage_bytes = p->stage_bytes;
  kp.b_bytes = 2 * p->NT * p->kc * 128;
  kp.a_swizzle_mode = p->kc == 64 ? 2 : 4;
  kp.acc_cols = 128 * p->NT;
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
  kp.entry_rows = p->d_entry_rows;
  kp.n_acc = p->n_acc;
  p->kp_valid = true;
  p->kp_a = A->values;
  p->kp_b = B;
  p->kp_c = C;
  p->kp_ldb = ldb;
  p->kp_ldc = ldc;
  set_peers(kp);
  select_split_counters(p, kp);
  kern<<<p->grid, kRsThreads, p->smem_bytes, stream>>>(kp);
  return cuda_check(cudaGetLastError(), "spmm rowstack kernel launch");
}

}  // namespace bsp
