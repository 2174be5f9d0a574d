// Fused block-sparse attention step on sm_100a tensor cores, one head:
//   O = softmax_rows(scale * Q K^T restricted to the mask's 32 x 32 blocks) V.
//
// This is the chain the reference runs as two separate programs with the
// probabilities in DRAM between them: its SDDMM (block_sddmm/kernels/compute/
// sddmm_block_multiply.cpp:72-193, golden bsr_matrix::sddmm,
// sparse_common/bsr_matrix.hpp:816-857) and its SpMM (block_spmm/kernels/
// compute/bmm_iter.cpp:92-185, golden bsr_matrix::spmm_bfloat16, 692-736),
// with the row softmax between them.  Here P never leaves the SM.
//
// Mapping (planner.cpp, plan_attn_host): a unit is 128 query rows (MMA M =
// four block-rows = the four TMEM lane quarters); its key blocks (the union of
// the four block-rows' mask columns) come four at a time ("chunks", 128 keys).
// Per chunk:
//   S   = Q K_c^T          MMA 128 x 128 x d into TMEM (double-buffered)
//   P   = exp2(S * scale * log2 e - m)   softmax warps, one thread per query
//         row: slots the row's block-row does not hold are masked out, the
//         running maximum m moves only when it grows by more than 2^8 (then
//         the O row and the row sum are rescaled), P is written to shared
//         memory as the K-major bf16 operand
//   O  += P V_c            MMA 128 x d x 128 into TMEM
// and at the end of the unit O / l is rounded to bf16 and stored.  The MMA
// warp issues S of chunk j + 1 before P V of chunk j, so the tensor pipe works
// while the softmax warps do.  K and V have separate two-slot rings (K of
// chunk j + 2 loads as soon as S of chunk j is done).
//
// Warp roles (256 threads, one CTA per SM):
//   warp 0      TMEM allocator + MMA issuer (converged warp, lane 0 issues)
//   warp 1      TMA: Q of each unit and the K chunks (one predicated
//               instruction: lane 2 s + h loads half h of key block slot s)
//   warp 2      TMA: the V chunks
//   warps 4..7  softmax, O rescale and epilogue (TMEM lane quarter = warp - 4)
// Every wait is bounded (bsp_ptx.cuh).
#include <cuda_bf16.h>

#include "bsp_internal.h"
#include "bsp_ptx.cuh"

namespace bsp {
using namespace dev;

namespace {

constexpr int kAtThreads = 8 * 32;
constexpr int kAtMmaWarp = 0;
constexpr int kAtKWarp = 1;
constexpr int kAtVWarp = 2;
constexpr int kAtSoft0 = 4;
constexpr uint32_t kAtPBytes = 128 * 128 * 2;  // one P tile
constexpr uint32_t kAtAtom = 128 * 128;        // 128 rows x 128 B (64 bf16 columns)
constexpr float kAtRescale = 8.0f;             // log2 of the growth that forces a rescale

struct AtSmemHeader {
  uint64_t q_full, q_empty;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], p_empty[2];
  uint64_t o_full, o_empty;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(AtSmemHeader) <= 1024, "header must fit its 1 KiB slot");

__host__ __device__ constexpr uint32_t at_tile(int d) { return 128u * static_cast<uint32_t>(d) * 2u; }

// Shared memory (from the 1 KiB-aligned base): header, Q, K[2], V[2], P[2].
struct AtLayout {
  uint32_t q, k[2], v[2], p[2];
  __device__ AtLayout(uint32_t base, int d) {
    const uint32_t t = at_tile(d);
    q = base + 1024u;
    k[0] = q + t;
    k[1] = k[0] + t;
    v[0] = k[1] + t;
    v[1] = v[0] + t;
    p[0] = v[1] + t;
    p[1] = p[0] + kAtPBytes;
  }
};

__device__ __forceinline__ uint32_t baddr(const uint64_t* b) { return smem_u32(b); }

__device__ __noinline__ bool at_drain_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl) {
  int zero = 0;
  WaitCtl c2{&zero, ctl.status, ctl.timeout_ns};
  return mbar_wait_bounded(bar, parity, c2, ST_TIMEOUT_DRAIN);
}

// Warp-converged bounded wait: true when every lane saw the phase complete.
__device__ __forceinline__ bool wait_all(uint32_t bar, uint32_t parity, const WaitCtl& ctl, uint32_t what) {
  return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, ctl, what));
}

// K (warp 1, with each unit's Q) or V (warp 2) producer.  Lane 2 s + h
// (< 4 * d / 64) loads the 32 x 64 box of half h of key block slot s.
template <bool kIsK>
__device__ __forceinline__ void at_producer(const AttnKernelParams& p, AtSmemHeader* hdr, const AtLayout& L,
                                           int u_begin, int u_end, const WaitCtl& ctl, int lane) {
  const int halves = p.d / 64;
  const int slot = lane / 2, half = lane & 1;
  const bool mine = lane < 2 * kAttnSlots && half < halves;
  const uint32_t tile = at_tile(p.d);
  const CUtensorMap* tm = kIsK ? &p.tm_k : &p.tm_v;
  uint64_t* full = kIsK ? hdr->k_full : hdr->v_full;
  uint64_t* empty = kIsK ? hdr->k_empty : hdr->v_empty;
  const uint32_t* buf = kIsK ? L.k : L.v;
  int64_t kn = 0;
  int qn = 0;
  uint32_t armed = 0, armed_parity = 0;
  bool ok = true;
#pragma unroll 1
  for (int u = u_begin; u < u_end && ok; ++u) {
    const int n = __ldg(&p.units[u].n_chunks);
    if (n == 0) continue;
    const int cb = __ldg(&p.units[u].chunk_begin);
    if (kIsK) {
      // Q of the unit, once the previous unit's last S MMA has read it
      ok = wait_all(baddr(&hdr->q_empty), static_cast<uint32_t>(qn & 1) ^ 1u, ctl, ST_TIMEOUT_PRODUCER);
      if (!ok) break;
      const int row0 = __ldg(&p.units[u].row0);
      mbar_arrive_expect_tx_pred(baddr(&hdr->q_full), tile, lane == 0);
      tma_load_2d_pred(L.q + static_cast<uint32_t>(lane) * kAtAtom, &p.tm_q, 64 * lane, row0,
                       baddr(&hdr->q_full), lane < halves);
      ++qn;
    }
    int32_t kb_next = mine ? __ldg(&p.chunks[cb].kb[slot]) : -1;
#pragma unroll 1
    for (int j = 0; j < n; ++j) {
      const int64_t g = kn + j;
      const int st = static_cast<int>(g & 1);
      const uint32_t ph = static_cast<uint32_t>((g >> 1) & 1);
      const int32_t kb = kb_next;
      if (j + 1 < n && mine) kb_next = __ldg(&p.chunks[cb + j + 1].kb[slot]);
      ok = wait_all(baddr(&empty[st]), ph ^ 1u, ctl, ST_TIMEOUT_PRODUCER);
      if (!ok) break;
      const uint32_t fb = baddr(&full[st]);
      mbar_arrive_expect_tx_pred(fb, tile, lane == 0);
      tma_load_2d_pred(buf[st] + static_cast<uint32_t>(half) * kAtAtom + static_cast<uint32_t>(slot) * 4096u, tm,
                       64 * half, kb >= 0 ? kb * 32 : -32, fb, mine);
      armed |= 1u << st;
      armed_parity = (armed_parity & ~(1u << st)) | (ph << st);
    }
    kn += n;
  }
  if (lane == 0) {
    for (int s = 0; s < 2; ++s)
      if (armed & (1u << s)) at_drain_wait(baddr(&full[s]), (armed_parity >> s) & 1u, ctl);
  }
  __syncwarp();
}

// MMA warp.
__device__ __forceinline__ void at_mma(const AttnKernelParams& p, AtSmemHeader* hdr, const AtLayout& L,
                                      uint32_t tmem_base, int u_begin, int u_end, const WaitCtl& ctl, int lane) {
  const uint32_t is0 = lane == 0 ? 1u : 0u;
  const int ks_d = p.d / 16;  // k-steps of S = Q K^T
  const uint32_t atom16 = kAtAtom >> 4;
  const uint64_t qdesc = smem_desc(L.q, 16u, 1024u, 2u);
  uint64_t kdesc[2], vdesc[2], pdesc[2];
  for (int s = 0; s < 2; ++s) {
    kdesc[s] = smem_desc(L.k[s], 16u, 1024u, 2u);
    vdesc[s] = smem_desc(L.v[s], kAtAtom, 1024u, 2u);  // MN-major: LBO = next 64 columns of d
    pdesc[s] = smem_desc(L.p[s], 16u, 1024u, 2u);
  }
  const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);
  const uint32_t idesc_pv = idesc_bf16_f32(128, p.d, 0, 1);
  const uint32_t t_o = tmem_base + 256u;
  int64_t kn = 0;
  int qn = 0, on = 0;
  bool ok = true;
  // O += P V of chunk g (acc: O already holds earlier chunks of the unit)
  auto pv = [&](int64_t g, bool acc) -> bool {
    const int st = static_cast<int>(g & 1);
    const uint32_t ph = static_cast<uint32_t>((g >> 1) & 1);
    if (!acc) {
      if (!wait_all(baddr(&hdr->o_empty), static_cast<uint32_t>(on & 1) ^ 1u, ctl, ST_TIMEOUT_MMA)) return false;
      ++on;
    }
    if (!wait_all(baddr(&hdr->v_full[st]), ph, ctl, ST_TIMEOUT_MMA)) return false;
    if (!wait_all(baddr(&hdr->p_full[st]), ph, ctl, ST_TIMEOUT_MMA)) return false;
    tc_fence_after();
#pragma unroll
    for (int k = 0; k < 8; ++k)
      mma_bf16_pred(t_o, pdesc[st] + (k >> 2) * atom16 + (k & 3) * 2u, vdesc[st] + k * 128u, idesc_pv,
                    acc || k > 0, is0);
    mma_commit_pred(baddr(&hdr->v_empty[st]), is0);
    mma_commit_pred(baddr(&hdr->p_empty[st]), is0);
    return true;
  };
#pragma unroll 1
  for (int u = u_begin; u < u_end && ok; ++u) {
    const int n = __ldg(&p.units[u].n_chunks);
    if (n == 0) continue;
    ok = wait_all(baddr(&hdr->q_full), static_cast<uint32_t>(qn & 1), ctl, ST_TIMEOUT_MMA);
    if (!ok) break;
    ++qn;
#pragma unroll 1
    for (int j = 0; j < n && ok; ++j) {
      const int64_t g = kn + j;
      const int st = static_cast<int>(g & 1);
      const uint32_t ph = static_cast<uint32_t>((g >> 1) & 1);
      ok = wait_all(baddr(&hdr->k_full[st]), ph, ctl, ST_TIMEOUT_MMA) &&
           wait_all(baddr(&hdr->s_empty[st]), ph ^ 1u, ctl, ST_TIMEOUT_MMA);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_s = tmem_base + static_cast<uint32_t>(st) * 128u;
#pragma unroll 1
      for (int k = 0; k < ks_d; ++k)
        mma_bf16_pred(t_s, qdesc + (k >> 2) * atom16 + (k & 3) * 2u, kdesc[st] + (k >> 2) * atom16 + (k & 3) * 2u,
                      idesc_s, k > 0, is0);
      mma_commit_pred(baddr(&hdr->s_full[st]), is0);
      mma_commit_pred(baddr(&hdr->k_empty[st]), is0);
      if (j == n - 1) mma_commit_pred(baddr(&hdr->q_empty), is0);
      if (j >= 1) ok = pv(g - 1, j > 1);
    }
    if (!ok) break;
    ok = pv(kn + n - 1, n > 1);
    if (!ok) break;
    mma_commit_pred(baddr(&hdr->o_full), is0);
    kn += n;
  }
  if (lane == 0) {
    mma_commit(baddr(&hdr->drain));
    at_drain_wait(baddr(&hdr->drain), 0, ctl);
  }
  __syncwarp();
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Softmax / rescale / epilogue warp of lane quarter q: thread = query row
// 32 q + lane of the unit.
__device__ __forceinline__ void at_softmax(const AttnKernelParams& p, AtSmemHeader* hdr, const AtLayout& L,
                                          uint8_t* gbase, uint32_t base, uint32_t tmem_base, int u_begin,
                                          int u_end, const WaitCtl& ctl, int warp, int lane) {
  const int q = warp - kAtSoft0;
  const int r = 32 * q + lane;  // row inside the unit
  const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
  const uint32_t t_o = lane_base + 256u;
  const int dc = p.d / 32;       // 32-column groups of a head row
  const float sl2 = p.scale_log2;
  int64_t kn = 0;
  int on = 0;
  bool ok = true;
#pragma unroll 1
  for (int u = u_begin; u < u_end && ok; ++u) {
    const int n = __ldg(&p.units[u].n_chunks);
    const int cb = __ldg(&p.units[u].chunk_begin);
    const int64_t row = static_cast<int64_t>(__ldg(&p.units[u].row0)) + r;
    uint4* orow = reinterpret_cast<uint4*>(p.o + row * p.ldo);
    if (n == 0) {
      if (row < p.S)
        for (int c = 0; c < p.d / 8; ++c) orow[c] = make_uint4(0, 0, 0, 0);
      continue;
    }
    float m_used = -INFINITY, l = 0.f;
    uint32_t bits_next = (__ldg(&p.chunks[cb].bits) >> (4 * q)) & 0xFu;
#pragma unroll 1
    for (int j = 0; j < n; ++j) {
      const int64_t g = kn + j;
      const int st = static_cast<int>(g & 1);
      const uint32_t ph = static_cast<uint32_t>((g >> 1) & 1);
      const uint32_t bits = bits_next;
      if (j + 1 < n) bits_next = (__ldg(&p.chunks[cb + j + 1].bits) >> (4 * q)) & 0xFu;
      ok = mbar_wait_bounded(baddr(&hdr->s_full[st]), ph, ctl, ST_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t t_s = lane_base + static_cast<uint32_t>(st) * 128u;
      // pass 1: the row maximum over the slots this block-row holds
      float mx = -INFINITY;
#pragma unroll 1
      for (int s = 0; s < kAttnSlots; ++s) {
        if (!((bits >> s) & 1u)) continue;  // warp-uniform
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_s + 32u * s, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, __uint_as_float(v[i]));
      }
      mx *= sl2;
      const bool need = mx > m_used + kAtRescale;
      if (__any_sync(0xffffffffu, need)) {
        const float new_m = need ? mx : m_used;
        const float alpha = need ? (m_used == -INFINITY ? 0.f : exp2f(m_used - new_m)) : 1.f;
        if (j >= 1) {
          // O holds the unit's chunks 0..j-1: wait for the last of those P V
          const int64_t gp = g - 1;
          ok = mbar_wait_bounded(baddr(&hdr->p_empty[gp & 1]), static_cast<uint32_t>((gp >> 1) & 1), ctl,
                                 ST_TIMEOUT_EPILOGUE);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < dc; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(t_o + 32u * c, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            tmem_st_32x32b_x32(t_o + 32u * c, v);
          }
          tmem_st_wait();
        }
        l *= alpha;
        m_used = new_m;
      }
      // pass 2: P = exp2(S * sl2 - m) into this chunk's P buffer
      ok = mbar_wait_bounded(baddr(&hdr->p_empty[st]), ph ^ 1u, ctl, ST_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      uint8_t* prow = gbase + (L.p[st] - base) + static_cast<uint32_t>(r) * 128u;
#pragma unroll 1
      for (int s = 0; s < kAttnSlots; ++s) {
        uint32_t w[16];
        if ((bits >> s) & 1u) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_s + 32u * s, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float a = exp2f(__uint_as_float(v[2 * i]) * sl2 - m_used);
            const float b = exp2f(__uint_as_float(v[2 * i + 1]) * sl2 - m_used);
            w[i] = pack_bf16(a, b);
            l += __uint_as_float(w[i] << 16) + __uint_as_float(w[i] & 0xFFFF0000u);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = 0u;
        }
        // keys 32 s .. 32 s + 31: atom s / 2, 16-byte chunks 4 (s & 1) .. + 3, XOR-swizzled by row
        uint8_t* atom = prow + static_cast<uint32_t>(s >> 1) * kAtAtom;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t chunk = static_cast<uint32_t>(4 * (s & 1) + c) ^ static_cast<uint32_t>(r & 7);
          *reinterpret_cast<uint4*>(atom + chunk * 16u) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(baddr(&hdr->s_empty[st]));
        mbar_arrive(baddr(&hdr->p_full[st]));
      }
    }
    if (!ok) break;
    // epilogue: O / l, rounded once to bf16
    ok = mbar_wait_bounded(baddr(&hdr->o_full), static_cast<uint32_t>(on & 1), ctl, ST_TIMEOUT_EPILOGUE);
    if (!__all_sync(0xffffffffu, ok)) break;
    ++on;
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
    for (int c = 0; c < dc; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_o + 32u * c, v);
      tmem_ld_wait();
      if (row < p.S) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          orow[4 * c + i] = make_uint4(pack_bf16(__uint_as_float(v[8 * i]) * inv, __uint_as_float(v[8 * i + 1]) * inv),
                                       pack_bf16(__uint_as_float(v[8 * i + 2]) * inv, __uint_as_float(v[8 * i + 3]) * inv),
                                       pack_bf16(__uint_as_float(v[8 * i + 4]) * inv, __uint_as_float(v[8 * i + 5]) * inv),
                                       pack_bf16(__uint_as_float(v[8 * i + 6]) * inv, __uint_as_float(v[8 * i + 7]) * inv));
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(baddr(&hdr->o_empty));
    kn += n;
  }
}

__global__ void __launch_bounds__(kAtThreads, 1) attn_tcgen05(const __grid_constant__ AttnKernelParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  AtSmemHeader* hdr = reinterpret_cast<AtSmemHeader*>(gbase);
  const AtLayout L(base, p.d);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int u_begin = p.cta_begin[blockIdx.x];
  const int u_end = p.cta_begin[blockIdx.x + 1];

  if (threadIdx.x == 32) {
    mbar_init(baddr(&hdr->q_full), 1);
    mbar_init(baddr(&hdr->q_empty), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(baddr(&hdr->k_full[s]), 1);
      mbar_init(baddr(&hdr->k_empty[s]), 1);
      mbar_init(baddr(&hdr->v_full[s]), 1);
      mbar_init(baddr(&hdr->v_empty[s]), 1);
      mbar_init(baddr(&hdr->s_full[s]), 1);
      mbar_init(baddr(&hdr->s_empty[s]), 4);
      mbar_init(baddr(&hdr->p_full[s]), 4);
      mbar_init(baddr(&hdr->p_empty[s]), 1);
    }
    mbar_init(baddr(&hdr->o_full), 1);
    mbar_init(baddr(&hdr->o_empty), 4);
    mbar_init(baddr(&hdr->drain), 1);
    hdr->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
  }
  if (warp == kAtMmaWarp) {
    tmem_alloc(smem_u32(&hdr->tmem_base), static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = hdr->tmem_base;
  const WaitCtl ctl{&hdr->abort_flag, p.status, p.timeout_ns};

  if (warp == kAtMmaWarp) {
    at_mma(p, hdr, L, tmem_base, u_begin, u_end, ctl, lane);
  } else if (warp == kAtKWarp) {
    at_producer<true>(p, hdr, L, u_begin, u_end, ctl, lane);
  } else if (warp == kAtVWarp) {
    at_producer<false>(p, hdr, L, u_begin, u_end, ctl, lane);
  } else if (warp >= kAtSoft0) {
    at_softmax(p, hdr, L, gbase, base, tmem_base, u_begin, u_end, ctl, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kAtMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
}

}  // namespace

int attn_smem_bytes(int d) { return static_cast<int>(2048u + 5u * at_tile(d) + 2u * kAtPBytes); }

bsp_status launch_attn(const bsp_attn_plan* p, const void* Q, int64_t ldq, const void* K, int64_t ldk,
                       const void* V, int64_t ldv, float scale, void* O, int64_t ldo, cudaStream_t stream) {
  if (p->n_units == 0) return BSP_OK;
  bsp_device* dev = p->dev;
  if (reinterpret_cast<uintptr_t>(O) % 16 || (ldo * 2) % 16)
    return set_error(BSP_ERR_INVALID_ARG, "O must be 16-byte aligned with a 16-byte row pitch");
  AttnKernelParams kp;
  memset(&kp, 0, sizeof(kp));
  bsp_status st = encode_2d(dev, &kp.tm_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Q, p->d, p->S, ldq, 64, 128,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == BSP_OK)
    st = encode_2d(dev, &kp.tm_k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, p->d, p->S, ldk, 64, 32,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == BSP_OK)
    st = encode_2d(dev, &kp.tm_v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, V, p->d, p->S, ldv, 64, 32,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != BSP_OK) return st;
  kp.units = p->d_units;
  kp.chunks = p->d_chunks;
  kp.cta_begin = p->d_cta_begin;
  kp.o = static_cast<uint16_t*>(O);
  kp.ldo = ldo;
  kp.status = dev->d_status;
  kp.timeout_ns = p->timeout_ns;
  kp.S = static_cast<int32_t>(p->S);
  kp.d = static_cast<int32_t>(p->d);
  kp.scale_log2 = scale * 1.4426950408889634f;
  kp.tmem_cols = p->tmem_cols;
  cudaError_t e = cudaFuncSetAttribute(attn_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize, p->smem_bytes);
  if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(attn)");
  attn_tcgen05<<<p->grid, kAtThreads, p->smem_bytes, stream>>>(kp);
  return cuda_check(cudaGetLastError(), "attention kernel launch");
}

}  // namespace bsp
