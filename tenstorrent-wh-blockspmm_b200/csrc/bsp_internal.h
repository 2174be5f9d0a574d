// Internal types shared by the host planner, the C ABI and the kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "bsp.h"

namespace bsp {

constexpr int kMaxGroupRows = 8;   // DDA row-group size limit
constexpr int kMaxNTiles = 4;      // SNF/DDA n-tiles per unit limit
constexpr int kTileN = 128;        // dense columns per MMA (MMA M dimension)
constexpr int kTmemCols = 512;     // TMEM columns per SM
constexpr int kSmemBudget = 227 * 1024;

// ---- SpMM schedule ----------------------------------------------------------
// One unit = a group of `nrows` consecutive block-rows x a sub-row slab of
// height Rs x `nt` consecutive 128-column tiles of C.  Its steps (one per
// distinct column of the group, in order) list, per member row, the block to
// multiply (or -1).
struct SpmmUnit {
  int32_t row0;        // first block-row of the group
  int32_t nrows;       // block-rows in the group (1..G)
  int32_t r_off;       // first row of the Rs-high slab inside each block
  int32_t n0;          // first column of C covered
  int32_t nt;          // 128-column tiles covered (1..NT)
  int32_t step_begin;  // steps [step_begin, step_end) in the step table
  int32_t step_end;
  int32_t row_mask;    // bit g: block-row row0+g has at least one block
};
static_assert(sizeof(SpmmUnit) == 32, "unit layout");

constexpr int kMaxPeers = 7;   // one node: up to 8 GPUs

struct SpmmKernelParams {
  CUtensorMap tm_a;  // A values as [nnzb*R rows, C cols] bf16, box {kc, Rs}
  CUtensorMap tm_b;  // B: 3-D {64 cols, K rows, N/64 blocks} box {64, kc, 2*NT}
                     // (b3d) or 2-D [K rows, N cols] box {64, kc}; 128B swizzle
  const SpmmUnit* units;        // in CTA order
  const int32_t* cta_begin;     // [grid + 1]
  const int32_t* steps;         // [nsteps][1 + G]: col, blk[G]
  unsigned int* status;
  uint64_t timeout_ns;
  void* c_ptr;                  // C, row-major
  int64_t ldc;                  // C leading dimension (elements)
  int32_t R, C, Rs, kc, nkc, G, NT, step_stride;
  int32_t c_f32;                // C element type is f32
  int32_t stages;               // pipeline depth
  int32_t stage_bytes;          // bytes per pipeline stage (1024-aligned)
  int32_t b_bytes;              // bytes of the B part of a stage (NT tiles)
  int32_t a_swizzle_mode;       // descriptor layout code of the A chunk (2 = 128B, 4 = 64B)
  int32_t acc_cols;             // TMEM columns of one accumulator set (NT*G*Rs)
  int32_t tmem_cols;            // TMEM columns allocated
  int32_t N;                    // C columns
  int32_t stacked;              // DDA: one MMA over the group's stacked blocks
  int32_t nprod;                // producer warps issuing stages round-robin
  int32_t b3d;                  // tm_b is the 3-D view (one box per step)
  const int4* stage_list;       // row-stacked kernel: per-CTA pipeline stages (4 x int4 each)
  const int32_t* cta_stage_begin;  // [grid + 1]
  int32_t sub_bytes;            // row-stacked: bytes of one sub-step (B slice + entry slots)
  // Replicated output (row-stacked kernel): every C store is repeated into the
  // n_peers other GPUs' C buffers (peer pointers mapped over NVLink, same
  // layout and ldc), fusing the row-panel all-gather into the epilogue.
  int32_t n_peers;
  void* peer_c[kMaxPeers];
  // byte offset (from the 1 KiB-aligned shared-memory base) of a 16 KiB area
  // where each epilogue warp stages 32 rows x 128 bytes of C, so that peer
  // stores leave as whole 128-byte lines; 0 = no area (16-byte peer stores)
  int32_t xfer_off;
  // split-K (row-stacked kernels): a unit with nt & 0xFF = n parts > 1 is part
  // (nt >> 8) & 0xFF of n; its partial tile goes to workspace slot r_off + part
  // (acc_cols / 4 float4 columns of 128 rows), and the part that takes the
  // last count of split_counters[r_off] sums the n partials and stores C.
  // The plan holds two counter sets used by alternate launches: every launch
  // zeroes the other set (split_counters_next, n_split_counters entries) before
  // any of its waits, so a launch that gave up after a timeout, with counts
  // left behind, cannot disturb the launch after next.
  float* split_ws;
  int32_t* split_counters;
  int32_t* split_counters_next;
  int32_t n_split_counters;
  // Testing only (bsp_testing_spmm_drop_stage): k + 1 makes CTA 0's producer
  // leave its k-th pipeline stage unissued (no copy, no arrive), so that the
  // MMA warp's bounded wait on it runs out; 0 = off.
  int32_t debug_drop_stage;
  // Accumulators in TMEM: 1 = one of acc_cols columns (wide units of 512
  // columns), anything else = two (double-buffered, acc_cols each).
  int32_t n_acc;
  // Row-stacked kernel: stacking order of the block-rows.  Entry e of the
  // stack (unit row0 + g) is block-row entry_rows[e]; nullptr = identity.
  const int32_t* entry_rows;
};

// Row-stacked kernel stage descriptor (16 words), precomputed by the planner
// so that a producer warp issues a stage without arithmetic or dependent
// loads.  A stage carries one or two "sub-steps" (consecutive block-columns of
// the same unit), each a B slice plus the entries' blocks.
//   w[0] flags: bits 0-3 / 4-7 entries present in sub-step 0 / 1,
//        8-11 / 12-15 entry slots of sub-step 0 / 1 to zero first,
//        16-19 present blocks in total, RS_F_* bits below
//   w[1] bz: first 64-column block of the unit (3-D map) or first column (2-D)
//   w[2] ax: A column coordinate (k-chunk offset)
//   w[3], w[4] ky: B row coordinate of sub-step 0, 1 (block column * C + k offset)
//   w[5..8], w[9..12] ay[g]: A row of entry g's block slab in sub-step 0, 1 (or -1)
enum : int32_t {
  RS_F_FIRST = 1 << 24,  // first stage of a unit
  RS_F_LAST = 1 << 25,   // last stage of a unit
  RS_F_EMPTY = 1 << 26,  // unit without blocks: nothing to load or multiply
  RS_F_TWO = 1 << 27,    // the stage carries two sub-steps
};
constexpr int kRsStageWords = 16;

// Twin stage descriptor (CTA-pair kernel, variant 3): a stage is one
// block-column of a twin, two pair units (a: entries 0..3, b: 4..7 of this
// CTA) of the same column tile stepping through the union of their columns
// and sharing each B slice.
//   w[0] flags: bits 0-7 entry slots to load (present block or zero box),
//        TW_F_* bits below
//   w[1] bz: first 64-column block of this CTA's half of the tile
//   w[3] ky: B row of the block-column (column * 32)
//   w[4..11] ay[s]: A row of slot s's block slab, or -32 (zero box)
enum : int32_t {
  TW_F_MMA_A = 1 << 8,     // unit a multiplies at this stage
  TW_F_MMA_B = 1 << 9,     // unit b multiplies at this stage
  TW_F_FIRST_A = 1 << 16,  // first stage of unit a (its accumulator starts)
  TW_F_LAST_A = 1 << 17,   // last stage of unit a (its accumulator is complete)
  TW_F_FIRST_B = 1 << 18,
  TW_F_LAST_B = 1 << 19,
  TW_F_EMPTY = 1 << 20,    // nothing to load or multiply (both units without blocks)
};
// Unit record flag (SpmmUnit::nt bit 16): this split-K part of the unit never
// multiplies, its accumulator holds nothing of the unit, its partial is zero.
constexpr int32_t kUnitNoAcc = 1 << 16;

// ---- SDDMM schedule ---------------------------------------------------------
// One unit = one block-row slab (Rs rows) x up to 4 output segments, each 32
// consecutive output columns of one mask block.
struct SddmmUnit {
  int32_t row;        // block-row i
  int32_t r_off;      // first row of the Rs-high slab
  int32_t nseg;       // valid segments (1..4)
  int32_t pad;
  int32_t blk[4];     // mask block index of each segment
  int32_t col[4];     // absolute first column (j*C + c0) of each segment
};
static_assert(sizeof(SddmmUnit) == 48, "unit layout");

// Row-stacked SDDMM work unit: 128 consecutive output rows (4 slabs of 32,
// one TMA box of A) against up to 8 gathered 32-column segments of B.  The
// MMA computes the full 128 x (32 * nseg) tile; the epilogue keeps the
// (slab, segment) pairs that the mask holds.
constexpr int kSddmmRsMaxSeg = 8;
struct SddmmRsUnit {
  int32_t row0;                   // first output row (a multiple of 128)
  int32_t nseg;                   // segments used (1..8)
  int32_t pad[2];
  int32_t seg_col[kSddmmRsMaxSeg];  // first column of each segment (j*C + c0), -1 unused
  int32_t blk[4][kSddmmRsMaxSeg];   // mask block holding (slab q, segment s), -1 none
};
static_assert(sizeof(SddmmRsUnit) == 176, "unit layout");

struct SddmmKernelParams {
  CUtensorMap tm_a;  // A [M rows, K cols] bf16, box {kc, Rs}
  CUtensorMap tm_b;  // B [K rows, N cols] bf16, box {32, kc}, 64B swizzle
  const SddmmUnit* units;
  const int32_t* cta_begin;
  const uint16_t* mask_vals;  // may be null
  uint16_t* out_vals;
  unsigned int* status;
  uint64_t timeout_ns;
  int32_t R, C, Rs, kc, nkc;
  int32_t stages, stage_bytes, a_bytes;
  int32_t a_swizzle_mode;
  int32_t tmem_cols;
  int32_t keep_a;  // DDA: A slab of the row stays resident across units of a row run
  // row-stacked variant
  const SddmmRsUnit* rs_units;
  int32_t M, nseg_max, nprod, seg_bytes;
};

// ---- SpGEMM schedule ------------------------------------------------------------
// C_bsr = A_bsr (Ra x Ca blocks) * B_bsr (Ca x Cb blocks).  A work unit is four
// "entries" (32-row slabs of output block-rows: MMA M = 128) against up to
// eight gathered 32-column "segments" of output block-columns (MMA N = 256).
// Its steps walk the shared block index k: each step stacks, per entry, the
// slab of A[i_e, k] (or a zero box) and gathers, per segment, the 32 columns
// of B[k, j_s] (or a zero box).  The product accumulates in TMEM over the
// unit's steps; the epilogue writes the (entry, segment) tiles whose output
// block exists.
constexpr int kSpgemmEnt = 4;
constexpr int kSpgemmMaxSeg = 8;
struct SpgemmUnit {
  int32_t step_begin;                 // first record in the step table
  int32_t n_steps;                    // >= 1
  int32_t n_ent;                      // entries in use (1..4)
  int32_t nseg;                       // segments in use (1..8)
  int32_t seg_x[kSpgemmMaxSeg];       // column of segment s inside its block (t*32); 0 unused
  int32_t ent_r[kSpgemmEnt];          // row of entry e's slab inside its block (slab*32)
  int32_t out_blk[kSpgemmEnt][kSpgemmMaxSeg];  // output block of tile (e, s), -1 none
};
static_assert(sizeof(SpgemmUnit) == 192, "unit layout");

// One step = the TMA boxes that fill its operand slots.  Consecutive slots
// whose data is contiguous in memory (or which are all absent, i.e. zero)
// share one box of 1, 2, 4 (entries) or 1, 2, 4, 8 (segments) slots.
//   a_y[i]    box i of the entries: first row of A viewed as [nnzb_a*Ra, Ca]
//             (block * Ra + slab * 32), or -32*L for L zero slabs
//   b_z[i]    box i of the segments: first block of B viewed as
//             [nnzb_b][Ca][Cb], or -L for L zero segments
//   a_meta[i], b_meta[i]: bit 7 box present, bits 0-2 first slot,
//             bits 3-4 log2 of the slot count, bits 5-6 (segments) the
//             32-column slice t inside the block (x = 32 t)
struct SpgemmStep {
  int32_t a_y[kSpgemmEnt];
  int32_t b_z[kSpgemmMaxSeg];
  uint8_t a_meta[kSpgemmEnt];
  uint8_t b_meta[kSpgemmMaxSeg];
  uint8_t pad[4];
};
static_assert(sizeof(SpgemmStep) == 64, "step layout");
constexpr int kSpgemmBoxValid = 0x80;

struct SpgemmKernelParams {
  CUtensorMap tm_a[3];  // A values [nnzb_a*Ra rows, Ca cols], box {kc, 32 << l}
  CUtensorMap tm_b[4];  // B values [nnzb_b][Ca][Cb], box {32, kc, 1 << l}, 64B swizzle
  const SpgemmUnit* units;   // in CTA order
  const SpgemmStep* steps;
  const int32_t* cta_begin;  // [grid + 1]
  uint16_t* out_vals;
  unsigned int* status;
  uint64_t timeout_ns;
  int32_t Ra, Cb, kc, nkc;
  int32_t sps;               // sub-steps (step, k-chunk) per pipeline stage
  int32_t stages, stage_bytes, sub_bytes, a_slot, seg_bytes;
  int32_t a_swizzle_mode;    // 2 = 128B (kc 64), 4 = 64B (kc 32)
  int32_t tmem_cols, nseg_max, nprod;
};

// ---- fused attention step schedule -------------------------------------------
// O = softmax_rows(scale * Q K^T on the mask's blocks) V for one head.  A work
// unit is 128 query rows (four 32-row block-rows: MMA M); its key blocks are
// the union of those block-rows' mask columns, taken four at a time
// ("chunks": 128 keys = MMA N of S = Q K^T and MMA K of O += P V).  bits says
// which (block-row, key block) pairs of the chunk the mask holds; the others
// are masked to -inf before the softmax.
constexpr int kAttnSlots = 4;
constexpr int kAttnMaxParts = 16;
// A unit whose chunk list is much longer than the average CTA's share is cut
// into parts (consecutive chunk ranges) that run on different CTAs; each part
// writes its unnormalised O rows, running maxima and row sums to a workspace
// slot, and the part that finishes last (a counter per unit) merges them.
struct AttnUnit {
  int32_t row0;          // first query row (multiple of 128)
  int32_t chunk_begin;   // first chunk record of this part
  int32_t n_chunks;      // 0: no block-row of the unit holds a mask block (O rows = 0)
  int32_t n_parts;       // parts of the unit (1: not split)
  int32_t part;          // this part's index
  int32_t slot0;         // workspace slot of part 0 (parts use slot0 .. slot0 + n_parts - 1)
  int32_t counter;       // index of the unit's completion counter
  int32_t pad;
};
static_assert(sizeof(AttnUnit) == 32, "unit layout");
struct AttnChunk {
  int32_t kb[kAttnSlots];  // key block of each slot, -1 none (zero box)
  uint32_t bits;           // bit 4 q + s: block-row q of the unit holds key block kb[s]
  int32_t pad[3];
};
static_assert(sizeof(AttnChunk) == 32, "chunk layout");

struct AttnKernelParams {
  CUtensorMap tm_q;  // Q [S, d], box {64, 128}, 128B swizzle
  CUtensorMap tm_k;  // K [S, d], box {64, 32}
  CUtensorMap tm_v;  // V [S, d], box {64, 32}
  const AttnUnit* units;
  const AttnChunk* chunks;
  const int32_t* cta_begin;
  uint16_t* o;
  int64_t ldo;
  unsigned int* status;
  uint64_t timeout_ns;
  float* work;           // split units: per slot 128 x d partial O, then 128 maxima, 128 sums
  int32_t* counters;     // split units: parts finished (the merging part resets it to 0)
  int32_t* counters_next;  // the other launch parity's counters, zeroed by this launch
  int32_t n_counters;
  int32_t S, d;
  float scale_log2;      // softmax scale * log2(e)
  int32_t tmem_cols;
};

// ---- host objects -------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace bsp

struct bsp_device {
  int ordinal = 0;
  int sm_count = 0;
  int max_smem_optin = 0;
  unsigned int* d_status = nullptr;  // device status word(s)
  bsp::PFN_encodeTiled encode = nullptr;
  // grow-only workspace for the host-buffer entry points
  void* ws = nullptr;
  size_t ws_bytes = 0;
  void* pinned = nullptr;
  size_t pinned_bytes = 0;
  // host-buffer entry points: plan tables of their temporary plans (device
  // area + pinned staging, grow-only) and copy / compute streams
  void* plan_ws = nullptr;
  size_t plan_ws_bytes = 0;
  void* aux_ws = nullptr;   // attention merge workspace of host-buffer plans
  size_t aux_ws_bytes = 0;
  cudaStream_t s_h2d = nullptr, s_comp = nullptr, s_d2h = nullptr;
  std::vector<cudaEvent_t> ev_in, ev_out;
  // bsp_spmm_host_batch: per job slot, a grow-only device area for the plan
  // tables and split-K partials and a pinned staging area for the tables
  struct BatchSlot {
    void* d = nullptr;
    size_t d_bytes = 0;
    void* h = nullptr;
    size_t h_bytes = 0;
  };
  std::vector<BatchSlot> batch_slots;
};

struct bsp_spgemm_plan {
  bsp_device* dev = nullptr;
  int64_t M = 0, K = 0, N = 0, nnzb_a = 0, nnzb_b = 0;
  int32_t Ra = 0, Ca = 0, Cb = 0, kc = 0, nkc = 1, sps = 1;
  int32_t grid = 0, stages = 0, stage_bytes = 0, sub_bytes = 0, smem_bytes = 0, tmem_cols = 0;
  int32_t nseg_max = 8, nprod = 1;
  int32_t la_log2 = 0, lb_log2 = 0;  // largest box (log2 slots) of the entries / segments
  int64_t n_units = 0, n_steps = 0;
  int64_t n_boxes = 0;       // TMA boxes over all steps (one k-chunk)
  int64_t pairs = 0;         // block products A[i,k] * B[k,j] (useful work)
  uint64_t timeout_ns = 0;
  void* d_blob = nullptr;    // units | steps | cta_begin
  size_t blob_bytes = 0;
  bool blob_borrowed = false;  // tables live in the device's plan area (host-buffer path)
  bsp::SpgemmUnit* d_units = nullptr;
  bsp::SpgemmStep* d_steps = nullptr;
  int32_t* d_cta_begin = nullptr;
  // output pattern (host), sorted columns per block-row
  std::vector<int32_t> out_row_ptr, out_col_idx;
  std::vector<bsp::SpgemmUnit> h_units;
  std::vector<bsp::SpgemmStep> h_steps;
  std::vector<int32_t> h_cta_begin;
};

struct bsp_attn_plan {
  bsp_device* dev = nullptr;
  int64_t S = 0, d = 0, nnzb = 0;
  int64_t mask_blocks = 0;   // distinct (block-row, key block) pairs (useful work)
  int32_t grid = 0, smem_bytes = 0, tmem_cols = 0;
  int64_t n_units = 0, n_chunks = 0;
  int64_t n_slots = 0, n_counters = 0;  // workspace slots and counters of split units
  uint64_t timeout_ns = 0;
  void* d_blob = nullptr;    // units | chunks | cta_begin | 2 x counters (zeroed)
  size_t blob_bytes = 0;
  bool blob_borrowed = false;  // tables and merge workspace belong to the device (host-buffer path)
  float* d_work = nullptr;
  bsp::AttnUnit* d_units = nullptr;
  bsp::AttnChunk* d_chunks = nullptr;
  int32_t* d_cta_begin = nullptr;
  int32_t* d_counters = nullptr;  // two sets of n_counters, alternate launches
  mutable uint32_t launch_parity = 0;
  std::vector<bsp::AttnUnit> h_units;
  std::vector<bsp::AttnChunk> h_chunks;
  std::vector<int32_t> h_cta_begin;
};

struct bsp_spmm_plan {
  bsp_device* dev = nullptr;
  int64_t M = 0, K = 0, N = 0, nnzb = 0;
  int32_t R = 0, C = 0, Rs = 0, kc = 0, G = 1, NT = 1, stacked = 0;
  bsp_dtype c_type = BSP_BF16;
  bsp_strategy strategy = BSP_NAIVE;
  int32_t grid = 0, stages = 0, stage_bytes = 0, smem_bytes = 0, tmem_cols = 0, nprod = 1;
  int32_t variant = 0;      // 0: swap-AB kernel (spmm.cu), 1: row-stacked kernel (spmm_rowstack.cu)
  int32_t nsub = 1, sub_bytes = 0;  // row-stacked: sub-steps per stage and their size
  int32_t xfer_off = 0;     // row-stacked: shared-memory staging area for peer stores (0: none)
  int32_t step_stride = 2;  // int32 words per step-table entry (1 + G)
  int64_t n_units = 0, n_steps = 0;
  // split-K (row-stacked kernels): units cut into parts whose partial tiles
  // meet in a workspace of n_split_slots tiles (128 rows x acc columns fp32)
  int64_t n_split_slots = 0;
  int32_t split_units = 0;
  float* d_split_ws = nullptr;       // owned unless blob_borrowed
  int32_t* d_split_counters = nullptr;  // in the blob (zeroed): two sets of one per slot
  mutable uint32_t launch_parity = 0;   // which counter set the next launch uses
  int32_t debug_drop_stage = 0;         // testing only, see SpmmKernelParams
  int32_t n_acc = 2;                    // row-stacked: TMEM accumulators (1: wide units)
  std::vector<int32_t> h_entry_rows;    // row-stacked: stacking order (empty = identity)
  int32_t* d_entry_rows = nullptr;      // in the blob
  uint64_t timeout_ns = 0;
  void* d_blob = nullptr;  // units | cta_begin | steps
  size_t blob_bytes = 0;
  bool blob_borrowed = false;  // tables live in the device's plan area (host-buffer path)
  bsp::SpmmUnit* d_units = nullptr;
  int32_t* d_cta_begin = nullptr;
  int32_t* d_steps = nullptr;
  int4* d_stage_list = nullptr;
  int32_t* d_cta_stage_begin = nullptr;
  // host copies (tests and the no-allocation variant reuse them)
  std::vector<bsp::SpmmUnit> h_units;
  std::vector<int32_t> h_cta_begin;
  std::vector<int32_t> h_steps;
  std::vector<int32_t> h_stage_list;       // row-stacked kernel: 16 words per stage
  std::vector<int32_t> h_cta_stage_begin;  // row-stacked kernel
  // launch cache: kernel parameters (tensor maps) for the last operand set
  mutable bool kp_valid = false;
  mutable bool attr_set = false;
  mutable const void* kp_a = nullptr;
  mutable const void* kp_b = nullptr;
  mutable const void* kp_c = nullptr;
  mutable int64_t kp_ldb = 0, kp_ldc = 0;
  mutable bsp::SpmmKernelParams kp;
};

struct bsp_sddmm_plan {
  bsp_device* dev = nullptr;
  int64_t M = 0, N = 0, K = 0, nnzb = 0;
  int32_t R = 0, C = 0, Rs = 0, kc = 0;
  bsp_strategy strategy = BSP_NAIVE;
  int32_t grid = 0, stages = 0, stage_bytes = 0, smem_bytes = 0, tmem_cols = 0, keep_a = 0;
  int64_t n_units = 0;
  uint64_t timeout_ns = 0;
  void* d_blob = nullptr;
  size_t blob_bytes = 0;
  bool blob_borrowed = false;  // tables live in the device's plan area (host-buffer path)
  bsp::SddmmUnit* d_units = nullptr;
  int32_t* d_cta_begin = nullptr;
  std::vector<bsp::SddmmUnit> h_units;
  std::vector<int32_t> h_cta_begin;
  // variant 1: row-stacked kernel (sddmm_rowstack.cu)
  int32_t variant = 0, nseg_max = 0, nprod = 0;
  bsp::SddmmRsUnit* d_rs_units = nullptr;
  std::vector<bsp::SddmmRsUnit> h_rs_units;
};

namespace bsp {
// error plumbing (capi.cpp)
bsp_status set_error(bsp_status s, const std::string& msg);
bsp_status cuda_check(cudaError_t e, const char* what);

// planners (planner.cpp); pure host logic, testable without a GPU
bsp_status plan_spmm_host(bsp_spmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                          int sm_count, int max_smem, const bsp_spmm_opts* opts);
bsp_status plan_sddmm_host(bsp_sddmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                           int sm_count, int max_smem, const bsp_sddmm_opts* opts);
void serpentine_order(const std::vector<int64_t>& weight, int parts,
                      std::vector<std::vector<int32_t>>* per_part);

// kernel launchers (spmm.cu / sddmm.cu)
bsp_status launch_spmm(const bsp_spmm_plan* p, const bsp_bsr_desc* A, const void* B, int64_t ldb,
                       void* C, int64_t ldc, cudaStream_t stream);
bsp_status launch_sddmm(const bsp_sddmm_plan* p, const bsp_bsr_desc* mask, const void* A,
                        int64_t lda, const void* B, int64_t ldb, void* out, cudaStream_t stream);
bsp_status launch_sddmm_rowstack(const bsp_sddmm_plan* p, const bsp_bsr_desc* mask, const void* A,
                                 int64_t lda, const void* B, int64_t ldb, void* out,
                                 cudaStream_t stream);
bsp_status plan_sddmm_rowstack(bsp_sddmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                               int sm_count, int max_smem, const bsp_sddmm_opts* opts);
int sddmm_rowstack_max_stages();
int sddmm_rowstack_max_producers();
bsp_status encode_2d(bsp_device* dev, CUtensorMap* tm, CUtensorMapDataType dt, int esize,
                     const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                     uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);
// rank-D tiled map; strides_bytes[rank-1] are the strides of dims 1..rank-1
bsp_status encode_nd(bsp_device* dev, CUtensorMap* tm, CUtensorMapDataType dt, int rank,
                     const void* ptr, const uint64_t* dims, const uint64_t* strides_bytes,
                     const uint32_t* box, CUtensorMapSwizzle swz);
int spmm_threads();
int spmm_max_producers();
int rowstack_max_producers();
int rowstack_max_stages();
bsp_status launch_spmm_rowstack(const bsp_spmm_plan* p, const bsp_bsr_desc* A, const void* B,
                                int64_t ldb, void* C, int64_t ldc, cudaStream_t stream,
                                void* const* peer_c = nullptr, int n_peers = 0);
// stage_lists false: units and per-CTA stage counts only (h_stage_list empty)
bsp_status plan_spmm_pair(bsp_spmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                          int sm_count, int max_smem, const bsp_spmm_opts* opts, bool stage_lists = true);
// twin units on CTA pairs (variant 3): 32 x 32-wide blocks (C == 32,
// R % 32 == 0) and N > 128; the caller falls back to plan_spmm_pair otherwise
bool spmm_twin_eligible(const bsp_spmm_plan* p);
bsp_status plan_spmm_twin(bsp_spmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                          int sm_count, int max_smem, const bsp_spmm_opts* opts, bool stage_lists = true);
bsp_status launch_spmm_pair(const bsp_spmm_plan* p, const bsp_bsr_desc* A, const void* B, int64_t ldb,
                            void* C, int64_t ldc, cudaStream_t stream, void* const* peer_c = nullptr,
                            int n_peers = 0);
bsp_status plan_spgemm_host(bsp_spgemm_plan* p, const int32_t* a_rp, const int32_t* a_ci,
                            const int32_t* b_rp, const int32_t* b_ci, int sm_count, int max_smem,
                            const bsp_spmm_opts* opts);
bsp_status launch_spgemm(const bsp_spgemm_plan* p, const void* a_vals, const void* b_vals,
                         void* out_vals, cudaStream_t stream);
int spgemm_max_stages();
int spgemm_max_producers();
void spmm_plan_traffic(const bsp_spmm_plan& p, int64_t out[4]);
bsp_status plan_attn_host(bsp_attn_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                          int sm_count, int max_smem, const bsp_spmm_opts* opts);
bsp_status launch_attn(const bsp_attn_plan* p, const void* Q, int64_t ldq, const void* K, int64_t ldk,
                       const void* V, int64_t ldv, float scale, void* O, int64_t ldo,
                       cudaStream_t stream);
int attn_smem_bytes(int d);
// Cap on the threads the planner spawns from the calling thread (0 = none;
// inherited by the planner's own helper threads).
void set_planner_thread_cap(int cap);
bsp_status plan_spmm_rowstack(bsp_spmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                              int sm_count, int max_smem, const bsp_spmm_opts* opts, bool stage_lists = true);

// Split-K counters of the next launch of a row-stacked plan: the set of this
// launch's parity, and the other set, which the launch zeroes for the one after.
inline void select_split_counters(const bsp_spmm_plan* p, SpmmKernelParams& k) {
  const int64_t n = p->n_split_slots;
  const uint32_t par = p->launch_parity & 1u;
  k.n_split_counters = static_cast<int32_t>(n);
  k.split_counters = p->d_split_counters ? p->d_split_counters + par * n : nullptr;
  k.split_counters_next = p->d_split_counters ? p->d_split_counters + (par ^ 1u) * n : nullptr;
  k.debug_drop_stage = p->debug_drop_stage;
  p->launch_parity ^= 1u;
}
}  // namespace bsp
