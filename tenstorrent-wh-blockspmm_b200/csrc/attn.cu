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
//         the O row and the row sum are rescaled), P is stored to TMEM as
//         bf16 pairs (row m in lane m)
//   O  += P V_c            MMA 128 x d x 128 into TMEM, A = P read from TMEM
//                          (only V crosses shared memory, so this MMA is not
//                          held back by shared-memory bandwidth)
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
constexpr uint32_t kAtAtom = 128 * 128;        // 128 rows x 128 B (64 bf16 columns)
constexpr float kAtRescale = 8.0f;             // log2 of the growth that forces a rescale
constexpr int kAtSoftWarps = 4;                // one per TMEM lane quarter
// TMEM columns: S buffers 0..255 (two of 128 fp32), P buffers 256..383 (two
// of 64: 128 bf16 keys packed in pairs), O 384 .. 384 + d.
constexpr int kAtSBuf = 2;
constexpr uint32_t kAtPCol = 256;
constexpr uint32_t kAtOCol = 384;

struct AtSmemHeader {
  uint64_t q_full, q_empty;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[kAtSBuf], s_empty[kAtSBuf];
  uint64_t p_full[2], p_empty[2];
  uint64_t o_full, o_empty;
  uint64_t merge_bar;  // the softmax warps, split-unit merge
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int merge_flag;
};
static_assert(sizeof(AtSmemHeader) <= 1024, "header must fit its 1 KiB slot");

__host__ __device__ constexpr uint32_t at_tile(int d) { return 128u * static_cast<uint32_t>(d) * 2u; }

// Shared memory (from the 1 KiB-aligned base): header, Q, K[2], V[2].
struct AtLayout {
  uint32_t q, k[2], v[2];
  __device__ AtLayout(uint32_t base, int d) {
    const uint32_t t = at_tile(d);
    q = base + 1024u;
    k[0] = q + t;
    k[1] = k[0] + t;
    v[0] = k[1] + t;
    v[1] = v[0] + t;
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
  uint64_t kdesc[2], vdesc[2];
  for (int s = 0; s < 2; ++s) {
    kdesc[s] = smem_desc(L.k[s], 16u, 1024u, 2u);
    vdesc[s] = smem_desc(L.v[s], kAtAtom, 1024u, 2u);  // MN-major: LBO = next 64 columns of d
  }
  const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);
  const uint32_t idesc_pv = idesc_bf16_f32(128, p.d, 0, 1);
  const uint32_t t_o = tmem_base + kAtOCol;
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
    // A = P from TMEM: 16 keys (8 packed columns) per MMA
    const uint32_t t_p = tmem_base + kAtPCol + 64u * static_cast<uint32_t>(st);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      mma_bf16_ts_pred(t_o, t_p + 8u * k, vdesc[st] + k * 128u, idesc_pv, acc || k > 0, is0);
    mma_commit_pred(baddr(&hdr->v_empty[st]), is0);
    mma_commit_pred(baddr(&hdr->p_empty[st]), is0);
    return true;
  };
  // S of chunk j + 2 is issued before P V of chunk j (kAtSBuf S buffers), so
  // the softmax of a chunk has two MMA groups' time before its P V is due.
  constexpr int kLead = kAtSBuf - 1;
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
      const int sb = static_cast<int>(g % kAtSBuf);
      const uint32_t sph = static_cast<uint32_t>((g / kAtSBuf) & 1);
      ok = wait_all(baddr(&hdr->k_full[st]), ph, ctl, ST_TIMEOUT_MMA) &&
           wait_all(baddr(&hdr->s_empty[sb]), sph ^ 1u, ctl, ST_TIMEOUT_MMA);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_s = tmem_base + static_cast<uint32_t>(sb) * 128u;
#pragma unroll 1
      for (int k = 0; k < ks_d; ++k)
        mma_bf16_pred(t_s, qdesc + (k >> 2) * atom16 + (k & 3) * 2u, kdesc[st] + (k >> 2) * atom16 + (k & 3) * 2u,
                      idesc_s, k > 0, is0);
      mma_commit_pred(baddr(&hdr->s_full[sb]), is0);
      mma_commit_pred(baddr(&hdr->k_empty[st]), is0);
      if (j == n - 1) mma_commit_pred(baddr(&hdr->q_empty), is0);
      if (j >= kLead) ok = pv(g - kLead, j > kLead);
    }
    for (int j = n > kLead ? n - kLead : 0; j < n && ok; ++j) ok = pv(kn + j, j > 0);
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

__device__ __forceinline__ void store_row_bf16(uint4* dst, const float* v, float scale) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    dst[i] = make_uint4(pack_bf16(v[8 * i] * scale, v[8 * i + 1] * scale), pack_bf16(v[8 * i + 2] * scale, v[8 * i + 3] * scale),
                        pack_bf16(v[8 * i + 4] * scale, v[8 * i + 5] * scale),
                        pack_bf16(v[8 * i + 6] * scale, v[8 * i + 7] * scale));
}

// Softmax / rescale / epilogue warp of TMEM lane quarter q = warp - 4:
// thread = query row 32 q + lane of the unit; the chunk's S row is read from
// TMEM once into registers.
__device__ __forceinline__ void at_softmax(const AttnKernelParams& p, AtSmemHeader* hdr, const AtLayout& L,
                                          uint8_t* gbase, uint32_t base, uint32_t tmem_base, int u_begin,
                                          int u_end, const WaitCtl& ctl, int warp, int lane) {
  const int q = warp - kAtSoft0;
  const int r = 32 * q + lane;  // row inside the unit
  const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
  const uint32_t t_o = lane_base + kAtOCol;
  const int gd = p.d / 32;      // 32-column groups of O
  const float sl2 = p.scale_log2;
  int64_t kn = 0;
  int on = 0, mp = 0;
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
      const int sb = static_cast<int>(g % kAtSBuf);
      const uint32_t sph = static_cast<uint32_t>((g / kAtSBuf) & 1);
      const int st = static_cast<int>(g & 1);
      const uint32_t ph = static_cast<uint32_t>((g >> 1) & 1);
      const uint32_t bits = bits_next;  // bit s: slot s held by this block-row
      if (j + 1 < n) bits_next = (__ldg(&p.chunks[cb + j + 1].bits) >> (4 * q)) & 0xFu;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->s_full[sb]), sph, ctl, ST_TIMEOUT_EPILOGUE))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t t_s = lane_base + static_cast<uint32_t>(sb) * 128u;
      uint32_t v[kAttnSlots][32];
#pragma unroll
      for (int s_ = 0; s_ < kAttnSlots; ++s_)
        if ((bits >> s_) & 1u) tmem_ld_32x32b_x32(t_s + 32u * s_, v[s_]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(baddr(&hdr->s_empty[sb]));  // S is in registers now
      float mx = -INFINITY;
#pragma unroll
      for (int s_ = 0; s_ < kAttnSlots; ++s_)
        if ((bits >> s_) & 1u) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, __uint_as_float(v[s_][i]));
        }
      // The scaled scores below are rounded exactly like this maximum (no
      // fused multiply-add), so every exponent S * sl2 - m stays <= 8 even
      // when the scores are so large that one fp32 ulp exceeds 2^8.
      mx = __fmul_rn(mx, sl2);
      const bool need = mx > m_used + kAtRescale;
      if (__any_sync(0xffffffffu, need)) {
        const float new_m = need ? mx : m_used;
        const float alpha = need ? (m_used == -INFINITY ? 0.f : exp2f(m_used - new_m)) : 1.f;
        if (j >= 1) {
          // O holds the unit's chunks 0..j-1: wait for the last of those P V
          const int64_t gp = g - 1;
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->p_empty[gp & 1]),
                                                         static_cast<uint32_t>((gp >> 1) & 1), ctl,
                                                         ST_TIMEOUT_EPILOGUE))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < gd; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(t_o + 32u * c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_32x32b_x32(t_o + 32u * c, o);
          }
          tmem_st_wait();
        }
        l *= alpha;
        m_used = new_m;
      }
      // P = exp2(S * sl2 - m) into this chunk's P buffer
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->p_empty[st]), ph ^ 1u, ctl, ST_TIMEOUT_EPILOGUE))) {
        ok = false;
        break;
      }
      uint32_t w[kAttnSlots * 16];  // this row's 128 keys as bf16 pairs
#pragma unroll
      for (int s_ = 0; s_ < kAttnSlots; ++s_) {
        if ((bits >> s_) & 1u) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint32_t x =
                pack_bf16(exp2f(__fsub_rn(__fmul_rn(__uint_as_float(v[s_][2 * i]), sl2), m_used)),
                          exp2f(__fsub_rn(__fmul_rn(__uint_as_float(v[s_][2 * i + 1]), sl2), m_used)));
            w[16 * s_ + i] = x;
            l += __uint_as_float(x << 16) + __uint_as_float(x & 0xFFFF0000u);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) w[16 * s_ + i] = 0u;
        }
      }
      const uint32_t t_p = lane_base + kAtPCol + 64u * static_cast<uint32_t>(st);
      tmem_st_32x32b_x32(t_p, *reinterpret_cast<const uint32_t(*)[32]>(w));
      tmem_st_32x32b_x32(t_p + 32u, *reinterpret_cast<const uint32_t(*)[32]>(w + 32));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(baddr(&hdr->p_full[st]));
    }
    if (!ok) break;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(baddr(&hdr->o_full), static_cast<uint32_t>(on & 1), ctl,
                                                   ST_TIMEOUT_EPILOGUE)))
      break;
    ++on;
    tc_fence_after();
    const int n_parts = __ldg(&p.units[u].n_parts);
    if (n_parts == 1) {
      // epilogue: O / l, rounded once to bf16
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < gd; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(t_o + 32u * c, o);
        tmem_ld_wait();
        if (row < p.S) store_row_bf16(orow + 4 * c, reinterpret_cast<const float*>(o), inv);
      }
    } else {
      // A part of a split unit: its unnormalised O row, running maximum and
      // row sum go to this part's workspace slot; the part that finishes last
      // merges O = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p, its own O
      // still in TMEM.
      const int slot0 = __ldg(&p.units[u].slot0);
      const int part = __ldg(&p.units[u].part);
      const int cnt = __ldg(&p.units[u].counter);
      // Slot layout: O as d/4 float4 columns of 128 rows (float4 j of row r at
      // j * 128 + r, so a warp's access to one column is 512 contiguous
      // bytes), then the 128 running maxima and the 128 row sums.
      const int64_t slot_floats = 128 * static_cast<int64_t>(p.d + 2);
      const float* base0 = p.work + slot0 * slot_floats;
      float* ws = p.work + (slot0 + part) * slot_floats;
      float4* wcol = reinterpret_cast<float4*>(ws) + r;
#pragma unroll 1
      for (int c = 0; c < gd; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(t_o + 32u * c, o);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          __stcg(wcol + (8 * c + i) * 128, make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                                       __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3])));
      }
      __stcg(ws + 128 * p.d + r, m_used);
      __stcg(ws + 128 * p.d + 128 + r, l);
      // two rounds of the softmax warps' merge barrier (bounded waits): all
      // partial rows written and fenced, then the counter result published
      __threadfence();
      __syncwarp();
      if (lane == 0) mbar_arrive(baddr(&hdr->merge_bar));
      ok = mbar_wait_bounded(baddr(&hdr->merge_bar), static_cast<uint32_t>(mp & 1), ctl, ST_TIMEOUT_EPILOGUE);
      ++mp;
      if (!__all_sync(0xffffffffu, ok)) break;
      if (r == 0) hdr->merge_flag = atomicAdd(p.counters + cnt, 1) == n_parts - 1 ? 1 : 0;
      __syncwarp();
      if (lane == 0) mbar_arrive(baddr(&hdr->merge_bar));
      ok = mbar_wait_bounded(baddr(&hdr->merge_bar), static_cast<uint32_t>(mp & 1), ctl, ST_TIMEOUT_EPILOGUE);
      ++mp;
      if (!__all_sync(0xffffffffu, ok)) break;
      if (*reinterpret_cast<volatile int*>(&hdr->merge_flag)) {
        __threadfence();
        float mk[kAttnMaxParts], wk[kAttnMaxParts];
#pragma unroll
        for (int k = 0; k < kAttnMaxParts; ++k)
          mk[k] = (k < n_parts && k != part) ? __ldcg(base0 + k * slot_floats + 128 * p.d + r) : -INFINITY;
        float M = m_used;
#pragma unroll
        for (int k = 0; k < kAttnMaxParts; ++k) M = fmaxf(M, mk[k]);
        const float w_self = (M == -INFINITY || m_used == -INFINITY) ? 0.f : exp2f(m_used - M);
        float Lt = w_self * l;
#pragma unroll
        for (int k = 0; k < kAttnMaxParts; ++k) {
          wk[k] = (M == -INFINITY || mk[k] == -INFINITY) ? 0.f : exp2f(mk[k] - M);
          if (wk[k] != 0.f) Lt += wk[k] * __ldcg(base0 + k * slot_floats + 128 * p.d + 128 + r);
        }
        const float inv = Lt > 0.f ? 1.f / Lt : 0.f;
#pragma unroll 1
        for (int c = 0; c < gd; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(t_o + 32u * c, o);
          tmem_ld_wait();
          float acc[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] = w_self * __uint_as_float(o[i]);
          // two other parts per round trip to L2 (16 loads in flight)
#pragma unroll 1
          for (int k0 = 0; k0 < n_parts; k0 += 2) {
            const float w0 = wk[k0], w1 = k0 + 1 < n_parts ? wk[k0 + 1] : 0.f;
            const float4* src0 = reinterpret_cast<const float4*>(base0 + k0 * slot_floats) + (8 * c) * 128 + r;
            const float4* src1 = src0 + slot_floats / 4;
            float4 t0[8], t1[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              t0[i] = w0 != 0.f ? __ldcg(src0 + i * 128) : make_float4(0.f, 0.f, 0.f, 0.f);
              t1[i] = w1 != 0.f ? __ldcg(src1 + i * 128) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              acc[4 * i] += w0 * t0[i].x + w1 * t1[i].x;
              acc[4 * i + 1] += w0 * t0[i].y + w1 * t1[i].y;
              acc[4 * i + 2] += w0 * t0[i].z + w1 * t1[i].z;
              acc[4 * i + 3] += w0 * t0[i].w + w1 * t1[i].w;
            }
          }
          if (row < p.S) store_row_bf16(orow + 4 * c, acc, inv);
        }
        if (r == 0) p.counters[cnt] = 0;  // ready for the next launch
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
  // zero the other launch parity's counters (before any wait of this launch)
  if (p.counters_next != nullptr)
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n_counters; i += gridDim.x * blockDim.x)
      p.counters_next[i] = 0;

  if (threadIdx.x == 32) {
    mbar_init(baddr(&hdr->q_full), 1);
    mbar_init(baddr(&hdr->q_empty), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(baddr(&hdr->k_full[s]), 1);
      mbar_init(baddr(&hdr->k_empty[s]), 1);
      mbar_init(baddr(&hdr->v_full[s]), 1);
      mbar_init(baddr(&hdr->v_empty[s]), 1);
      mbar_init(baddr(&hdr->p_full[s]), kAtSoftWarps);
      mbar_init(baddr(&hdr->p_empty[s]), 1);
    }
    mbar_init(baddr(&hdr->o_full), 1);
    mbar_init(baddr(&hdr->o_empty), kAtSoftWarps);
    mbar_init(baddr(&hdr->merge_bar), kAtSoftWarps);
    for (int b = 0; b < kAtSBuf; ++b) {
      mbar_init(baddr(&hdr->s_full[b]), 1);
      mbar_init(baddr(&hdr->s_empty[b]), kAtSoftWarps);
    }
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

int attn_smem_bytes(int d) { return static_cast<int>(2048u + 5u * at_tile(d)); }

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
  kp.work = p->d_work;
  {
    // alternate counter sets by launch; this launch zeroes the other one
    const uint32_t par = p->launch_parity & 1u;
    kp.n_counters = static_cast<int32_t>(p->n_counters);
    kp.counters = p->d_counters ? p->d_counters + par * p->n_counters : nullptr;
    kp.counters_next = p->d_counters ? p->d_counters + (par ^ 1u) * p->n_counters : nullptr;
  }
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
  p->launch_parity ^= 1u;
  return cuda_check(cudaGetLastError(), "attention kernel launch");
}

}  // namespace bsp
