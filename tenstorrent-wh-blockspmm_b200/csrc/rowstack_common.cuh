// Shared pieces of the row-stacked SpMM kernels (single CTA: spmm_rowstack.cu,
// CTA pair with 2-SM MMAs: spmm_pair.cu): warp roles and limits, the
// shared-memory header, stage flags and the epilogue.
#pragma once
#include <cuda_bf16.h>

#include "bsp_internal.h"
#include "bsp_ptx.cuh"

namespace bsp {
namespace rs {
using namespace dev;

constexpr int kRsMmaWarp = 0;
constexpr int kRsProd0 = 1;
constexpr int kRsMaxProducers = 3;
constexpr int kRsEpi0 = 4;
constexpr int kRsThreads = 8 * 32;
constexpr int kRsMaxStages = 30;
constexpr int kRsN = 256;       // MMA N: dense columns per unit
constexpr int kRsMaxG = 4;      // entries per stack (128 / 32)

struct RsSmemHeader {
  uint64_t full[kRsMaxStages];
  uint64_t empty[kRsMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint64_t merge_bar;   // the epilogue warps, split-K merge
  uint32_t info[kRsMaxStages];
  uint32_t tmem_base;
  int abort_flag;
  int merge_flag;       // this part takes the last count: it stores the tile
};
static_assert(sizeof(RsSmemHeader) <= 1024, "header must fit its 1 KiB slot");

enum : uint32_t {
  RS_FIRST = static_cast<uint32_t>(RS_F_FIRST),
  RS_LAST = static_cast<uint32_t>(RS_F_LAST),
  RS_EMPTY = static_cast<uint32_t>(RS_F_EMPTY),
  RS_TWO = static_cast<uint32_t>(RS_F_TWO),
};

__device__ __forceinline__ uint32_t baddr(const uint64_t* b) { return smem_u32(b); }

// Zero the other launch parity's split-K counters (grid-stride, before any
// wait of this launch, so it completes even when the launch gives up later).
__device__ __forceinline__ void rs_clear_next_counters(const SpmmKernelParams& p) {
  if (p.split_counters_next == nullptr) return;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n_split_counters; i += gridDim.x * blockDim.x)
    p.split_counters_next[i] = 0;
}

static __device__ __noinline__ bool rs_drain_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl) {
  int zero = 0;
  WaitCtl c2{&zero, ctl.status, ctl.timeout_ns};
  return mbar_wait_bounded(bar, parity, c2, ST_TIMEOUT_DRAIN);
}

// Epilogue warp with TMEM lane quarter q: lanes 32q..32q+31 are output rows of
// entry g = 32q / Rs; each thread writes its row, 32 columns per TMEM load.
// acc_empty_leader: 0 = arrive on this CTA's acc_empty; otherwise the
// shared::cluster address of the pair leader's acc_empty[0] (CTA-pair kernel).
template <bool kF32>
__device__ __forceinline__ void rs_epilogue(const SpmmKernelParams& p, RsSmemHeader* hdr,
                                           uint32_t tmem_base, int u_begin, int u_end,
                                           const WaitCtl& ctl, int warp, int lane,
                                           uint32_t acc_empty_leader = 0) {
  const int q = warp & 3;
  const int g = (32 * q) / p.Rs;
  const int rrow = (32 * q) % p.Rs + lane;
  const int slabs = p.R / p.Rs;
  int acc = 0;
  uint32_t acc_phase = 0;
  // C (and its peer copies) leaves as whole 128-byte row segments: the
  // warp's 32 rows x 128 bytes are staged in shared memory (16-byte pieces
  // XOR-swizzled by row), then each store instruction writes 4 rows x 128
  // contiguous bytes.  A thread storing its own row directly would make every
  // warp store touch 32 lines with 16 bytes each, which costs ~4 us per
  // 128 x 256 tile and bounds the low-density launches.
  constexpr int kEsz = kF32 ? 4 : 2;
  constexpr int kChunksPerFlush = 128 / (32 * kEsz);  // 32-column chunks per 128-byte segment
  const bool staged = p.xfer_off > 0;
  uint4* xf = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(hdr) + p.xfer_off) + q * (32 * 8);
  const int lrow = 32 * q + lane;  // row of the unit's 128-row tile
  const int64_t slot_floats = 128 * static_cast<int64_t>(p.acc_cols);
  const int nchunk = p.acc_cols / 32;  // 32-column chunks of the unit's tile
  int mp = 0;                          // merge-barrier rounds
  SpmmUnit nxt;
  if (u_begin < u_end) nxt = p.units[u_begin];
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    const SpmmUnit un = nxt;
    if (u + 1 < u_end) nxt = p.units[u + 1];
    if (!mbar_wait_bounded(baddr(&hdr->acc_full[acc]), acc_phase, ctl, ST_TIMEOUT_EPILOGUE)) break;
    tc_fence_after();
    const bool present = g < un.nrows && ((un.row_mask >> g) & 1);
    // a split part that never multiplied leaves a zero partial (twin units)
    const bool acc_ok = present && !(un.nt & kUnitNoAcc);
    const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * p.acc_cols);
    // Split-K: every part leaves its partial tile in its workspace slot
    // (float4 j of row r at j * 128 + r: 512-byte warp accesses); the part
    // that takes the last count sums the parts' partials and stores C.
    const int n_parts = un.nt & 0xFF;
    const float* parts_ws = nullptr;
    bool store = true;
    if (n_parts > 1) {
      const int part = (un.nt >> 8) & 0xFF;
      float4* own = reinterpret_cast<float4*>(p.split_ws + (un.r_off + part) * slot_floats) + lrow;
#pragma unroll 1
      for (int c = 0; c < nchunk; ++c) {
        uint32_t v[32];
        if (acc_ok) {
          tmem_ld_32x32b_x32(t_acc + static_cast<uint32_t>(c * 32), v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0u;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
          __stcg(own + (8 * c + i) * 128, make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                                      __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])));
      }
      // two rounds of the epilogue warps' merge barrier (bounded waits): all
      // partial rows written and fenced, then the counter result published
      __threadfence();
      __syncwarp();
      if (lane == 0) mbar_arrive(baddr(&hdr->merge_bar));
      bool ok = mbar_wait_bounded(baddr(&hdr->merge_bar), static_cast<uint32_t>(mp & 1), ctl, ST_TIMEOUT_EPILOGUE);
      ++mp;
      if (!__all_sync(0xffffffffu, ok)) break;
      if (q == 0 && lane == 0) hdr->merge_flag = atomicAdd(p.split_counters + un.r_off, 1) == n_parts - 1 ? 1 : 0;
      __syncwarp();
      if (lane == 0) mbar_arrive(baddr(&hdr->merge_bar));
      ok = mbar_wait_bounded(baddr(&hdr->merge_bar), static_cast<uint32_t>(mp & 1), ctl, ST_TIMEOUT_EPILOGUE);
      ++mp;
      if (!__all_sync(0xffffffffu, ok)) break;
      store = *reinterpret_cast<volatile int*>(&hdr->merge_flag) != 0;
      if (store) {
        __threadfence();
        parts_ws = p.split_ws + un.r_off * slot_floats;
        if (q == 0 && lane == 0) p.split_counters[un.r_off] = 0;  // ready for the next launch
      }
    }
    if (store && g < un.nrows) {
      const int e = p.entry_rows ? __ldg(p.entry_rows + un.row0 + g) : un.row0 + g;
      const int64_t row = static_cast<int64_t>(e / slabs) * p.R + (e % slabs) * p.Rs + rrow;
#pragma unroll 1
      for (int c = 0; c < nchunk; ++c) {
        const int n = un.n0 + c * 32;
        if (n >= p.N) break;
        uint32_t v[32];
        if (parts_ws) {
          // the sum of the parts' partials, in part order: the loads of four
          // partials' chunk are in flight together (one L2 round trip each)
          float a[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) a[i] = 0.f;
          if (present) {
#pragma unroll 1
            for (int k0 = 0; k0 < n_parts; k0 += 4) {
              float4 t[4][8];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float4* src =
                    reinterpret_cast<const float4*>(parts_ws + (k0 + k) * slot_floats) + (8 * c) * 128 + lrow;
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  t[k][i] = k0 + k < n_parts ? __ldcg(src + i * 128) : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int k = 0; k < 4; ++k)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  a[4 * i] += t[k][i].x;
                  a[4 * i + 1] += t[k][i].y;
                  a[4 * i + 2] += t[k][i].z;
                  a[4 * i + 3] += t[k][i].w;
                }
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(a[i]);
        } else if (present) {
          tmem_ld_32x32b_x32(t_acc + static_cast<uint32_t>(c * 32), v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0u;
        }
        const int64_t eo = row * p.ldc + n;  // element offset, the same in every peer's C
        const int piece0 = (c % kChunksPerFlush) * (32 * kEsz / 16);  // first 16-byte piece of this chunk
        if constexpr (kF32) {
          float* dst = static_cast<float*>(p.c_ptr) + eo;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 val = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            if (!staged && n + 4 * i < p.N) {
              reinterpret_cast<uint4*>(dst)[i] = val;
#pragma unroll 1
              for (int pp = 0; pp < p.n_peers; ++pp)
                reinterpret_cast<uint4*>(static_cast<float*>(p.peer_c[pp]) + eo)[i] = val;
            }
            if (staged) xf[lane * 8 + ((piece0 + i) ^ (lane & 7))] = val;
          }
        } else {
          __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.c_ptr) + eo;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t w[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(v[8 * i + 2 * h]),
                                                              __uint_as_float(v[8 * i + 2 * h + 1]));
              w[h] = *reinterpret_cast<const uint32_t*>(&b2);
            }
            const uint4 val = make_uint4(w[0], w[1], w[2], w[3]);
            if (!staged && n + 8 * i < p.N) {
              reinterpret_cast<uint4*>(dst)[i] = val;
#pragma unroll 1
              for (int pp = 0; pp < p.n_peers; ++pp)
                reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.peer_c[pp]) + eo)[i] = val;
            }
            if (staged) xf[lane * 8 + ((piece0 + i) ^ (lane & 7))] = val;
          }
        }
        // flush the staged 128-byte segments after the segment's last chunk
        if (staged && (c % kChunksPerFlush == kChunksPerFlush - 1 || n + 32 >= p.N ||
                       c == nchunk - 1)) {
          __syncwarp();
          const int nseg0 = un.n0 + (c - c % kChunksPerFlush) * 32;  // first column of the segment
          const int64_t row_w = row - lane;                             // the warp's first row
          const int pc = lane & 7;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (lane >> 3);
            const int col = nseg0 + pc * (16 / kEsz);
            if (col < p.N && pc < (c % kChunksPerFlush + 1) * (32 * kEsz / 16)) {
              const uint4 val = xf[r * 8 + (pc ^ (r & 7))];
              const int64_t off = (row_w + r) * p.ldc + col;
              *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.c_ptr) + off * kEsz) = val;
#pragma unroll 1
              for (int pp = 0; pp < p.n_peers; ++pp)
                *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.peer_c[pp]) + off * kEsz) = val;
            }
          }
          __syncwarp();
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (acc_empty_leader) mbar_remote_arrive(acc_empty_leader + static_cast<uint32_t>(acc) * 8u);
      else mbar_arrive(baddr(&hdr->acc_empty[acc]));
    }
    if (p.n_acc != 1) acc ^= 1;
    if (acc == 0) acc_phase ^= 1u;
  }
  // peer stores are visible system-wide before this CTA retires
  if (p.n_peers > 0) __threadfence_system();
}

}  // namespace rs
}  // namespace bsp
