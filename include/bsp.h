/*
 * bsp.h -- C ABI of the B200 block-sparse SpMM / SDDMM library (libbsp.so).
 *
 * This is the drop-in boundary for the reference's block-sparse hot path
 * (salmanra/Tenstorrent-WH-BlockSpMM).  Every entry point below names the
 * reference interface it replaces (file:line inside the reference project).
 * Plain pointers and sizes only: no C++ or torch types cross this boundary.
 *
 * Layout (all row-major, bf16 = raw 16-bit brain-float bit patterns):
 *   BSR matrix  H x W with R x C blocks:
 *     row_ptr[H/R + 1] int32, col_idx[nnzb] int32,
 *     values[nnzb * R * C]: block b occupies values[b*R*C .. (b+1)*R*C), row-major.
 *     This is the reference's bsr_matrix (sparse_common/bsr_matrix.hpp:202-213)
 *     without the tt-metal tilize step (test_block_spmm.cpp:77-78): blocks are
 *     row-major, so no tilize/untilize is needed.
 *   Dense matrix: row-major with a leading dimension (elements).
 *
 * Requirements checked by every call (BSP_ERR_INVALID_ARG otherwise):
 *   R % 32 == 0, C % 32 == 0, H % R == 0, W % C == 0      (reference: TT_ASSERTs,
 *     block_spmm/inc/host_code/bsr_spmm_multicore_load_balanced_new_DM.cpp:67-69)
 *   N % 8 == 0, leading dimensions % 8 == 0 (bf16) / % 4 (f32),
 *   device pointers 16-byte aligned.
 *
 * Streams are passed as `void*` (a cudaStream_t; NULL = legacy default stream).
 * Execute calls are stream-ordered and asynchronous; device-side errors (a
 * kernel wait that timed out) are latched in the device and reported by
 * bsp_device_synchronize / bsp_device_get_error.  A plan whose units were
 * split (split-K SpMM, split attention units) keeps a workspace and counters
 * that one launch uses at a time: run a plan's launches on one stream.
 */
#ifndef BSP_H_
#define BSP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BSP_VERSION_MAJOR 0
#define BSP_VERSION_MINOR 1

/* Status codes.  The reference reports errors by TT_ASSERT/TT_THROW
 * exceptions (e.g. load_balanced_new_DM.cpp:67-69); the C ABI returns codes
 * and keeps a per-thread message (bsp_last_error_string). */
typedef enum bsp_status {
  BSP_OK = 0,
  BSP_ERR_INVALID_ARG = 1,
  BSP_ERR_UNSUPPORTED = 2,
  BSP_ERR_CUDA = 3,
  BSP_ERR_TIMEOUT = 4,   /* a bounded in-kernel wait gave up; see bsp_device_get_error */
  BSP_ERR_NCCL = 5,
  BSP_ERR_ALLOC = 6,
  BSP_ERR_STATE = 7
} bsp_status;

/* Dataflow strategies of the reference, re-expressed for one B200 CTA:
 *   NAIVE: each work unit (block-row x 128-column tile) loads its own A blocks
 *          and B slices.  Reference "Naive",
 *          block_spmm/inc/host_code/bsr_spmm_multicore_load_balanced_new_DM.cpp:6-536
 *          and block_sddmm/inc/host_code/bsr_sddmm_multicore_naive.cpp:6-352.
 *   SNF:   an A block is loaded once and multiplied against several 128-column
 *          tiles of B (the reuse that store-and-forward along a core row gives).
 *          Reference "SnF in0", block_spmm/inc/host_code/bsr_spmm_multicore_snf.cpp:16-781.
 *   DDA:   SNF plus: a B slice is loaded once and shared by every block-row of
 *          a row group that has a block in that column (the reuse that the
 *          chain of direct addressing gives).  Reference "SnF in0 + CDA in1",
 *          block_spmm/inc/host_code/bsr_spmm_multicore_snfin0_cdain1.cpp:8-843;
 *          for SDDMM the A row panel is kept on chip across a row's blocks,
 *          block_sddmm/inc/host_code/bsr_sddmm_multicore_CDA.cpp:28-490. */
typedef enum bsp_strategy { BSP_NAIVE = 0, BSP_SNF = 1, BSP_DDA = 2 } bsp_strategy;

typedef enum bsp_dtype { BSP_BF16 = 0, BSP_F32 = 1 } bsp_dtype;

/* A BSR matrix whose arrays live in device memory (caller-owned). */
typedef struct bsp_bsr_desc {
  int64_t rows;           /* H */
  int64_t cols;           /* W */
  int32_t R;              /* block rows */
  int32_t C;              /* block cols */
  int64_t nnzb;           /* number of stored blocks */
  const int32_t* row_ptr; /* device, rows/R + 1 entries */
  const int32_t* col_idx; /* device, nnzb entries */
  const void* values;     /* device, nnzb*R*C bf16 (may be NULL for an SDDMM mask) */
} bsp_bsr_desc;

/* Options.  Zero-initialise and set what you need; 0 means "library default". */
typedef struct bsp_spmm_opts {
  int32_t no_load_balance; /* 1: contiguous unit split, the reference's *_no_lb
                              variants (block_spmm/inc/host_code.hpp:113-161) */
  int32_t group_rows;      /* DDA swap-AB kernel: block-rows per row group (B-slice
                              sharing).  -1 turns off: split-K of long units (SpMM
                              row-stacked and pair kernels), the resident A tile
                              (SDDMM CDA / SnF), unit splitting (attention) */
  int32_t n_tiles;         /* SNF/DDA swap-AB: 128-column tiles per work unit
                              (A reuse).  DDA row-stacked kernel: 4 = wide
                              units of 512 columns in one accumulator (N a
                              multiple of 512; each A block loaded once per
                              512 columns), otherwise 256 */
  int32_t max_ctas;        /* cap on persistent CTAs (default: all SMs) */
  int32_t timeout_ms;      /* bound on every in-kernel wait (default 2000) */
  int32_t group_mma;       /* DDA: 0/1 (default) the planner's choice of the
                              row-stacked kernels; 2 one MMA per present block
                              (swap-AB); 4 single-CTA row stacks; 5 row stacks
                              on CTA pairs; 6 twin units on CTA pairs (two row
                              groups of one column tile share each B slice;
                              32-wide blocks and N > 128, else as 5) */
  int32_t producers;       /* TMA-issuing warps per CTA (default: as many as fit) */
  int32_t steps_per_stage; /* DDA: block-columns per pipeline stage, 1 or 2
                              (default 2 for 32-wide blocks, else 1) */
} bsp_spmm_opts;

typedef bsp_spmm_opts bsp_sddmm_opts;

/* ---- device context ---------------------------------------------------
 * Replaces the reference's IDevice* (tt-metal CreateDevice/CloseDevice,
 * block_spmm/src/test_block_spmm.cpp:52).  Holds SM count, the tensor-map
 * encoder and a small device status word written by the kernels. */
typedef struct bsp_device bsp_device;

bsp_status bsp_device_open(int ordinal, bsp_device** out);
bsp_status bsp_device_close(bsp_device* dev);
/* cudaDeviceSynchronize + read and clear the kernels' latched status word. */
bsp_status bsp_device_synchronize(bsp_device* dev);
/* Latched device status bits (0 = none) without clearing; stream-synchronous. */
bsp_status bsp_device_get_error(bsp_device* dev, uint32_t* bits);
int bsp_device_sm_count(const bsp_device* dev);

const char* bsp_last_error_string(void);
const char* bsp_status_string(bsp_status s);

/* ---- device storage -------------------------------------------------------
 * Device buffers: the reference's buffer helper sparse_common::MakeBuffer
 * (sparse_common/host_code_utils.cpp:5-18, a tt-metal DRAM or L1 buffer) and
 * its blocking EnqueueWriteBuffer / EnqueueReadBuffer
 * (block_spmm/inc/host_code/bsr_spmm_multicore_load_balanced_new_DM.cpp:
 * 140-144, 499-505).  alloc: `bytes` of device memory on dev (256-byte
 * aligned), free: release it; write / read: blocking host <-> device copies. */
bsp_status bsp_buffer_alloc(bsp_device* dev, int64_t bytes, void** ptr);
bsp_status bsp_buffer_free(bsp_device* dev, void* ptr);
bsp_status bsp_buffer_write(bsp_device* dev, void* dst_device, const void* src_host, int64_t bytes);
bsp_status bsp_buffer_read(bsp_device* dev, void* dst_host, const void* src_device, int64_t bytes);

/* A persistent device copy of a host BSR matrix (the reference uploads A's
 * blocks, indptr and indices into fresh buffers on every call,
 * load_balanced_new_DM.cpp:140-144 and 502-505; here one upload serves any
 * number of plans and executes).  Checks the pattern (row_ptr starts at 0,
 * ends at nnzb and never decreases; column indices in range), copies it with
 * the values (host_values NULL: a pattern-only SDDMM mask) into ONE device
 * allocation and fills *out: row_ptr at the allocation's start, col_idx and
 * the values each at a 256-byte boundary.  Synchronous.  Free it with
 * bsp_bsr_free, which releases the allocation and zeroes the descriptor;
 * pass it only descriptors that bsp_bsr_upload filled. */
bsp_status bsp_bsr_upload(bsp_device* dev, int64_t rows, int64_t cols, int32_t R, int32_t C, int64_t nnzb,
                          const int32_t* host_row_ptr, const int32_t* host_col_idx,
                          const uint16_t* host_values, bsp_bsr_desc* out);
bsp_status bsp_bsr_free(bsp_device* dev, bsp_bsr_desc* desc);

/* ---- SpMM: C[M x N] = A_bsr[M x K] * B[K x N] ---------------------------
 * Replaces HostCodeFunctionPtr (block_spmm/inc/host_code.hpp:165-177) and the
 * three planners behind it.  A plan is the reference planner's output (row
 * folding, serpentine load balance, tiling: load_balanced_new_DM.cpp:50-393)
 * for one sparsity pattern and one N; it owns a small device-side schedule.
 * Every element of C is written, including the rows of empty block-rows
 * (the reference leaves those to the caller's zero-initialised buffer,
 * load_balanced_new_DM.cpp:524-531). */
typedef struct bsp_spmm_plan bsp_spmm_plan;

/* host_row_ptr / host_col_idx: host copies of A's pattern; pass NULL to have
 * the plan copy them from A (synchronous D2H). */
bsp_status bsp_spmm_plan_create(bsp_device* dev, const bsp_bsr_desc* A, const int32_t* host_row_ptr,
                                const int32_t* host_col_idx, int64_t N, bsp_dtype c_type,
                                bsp_strategy strategy, const bsp_spmm_opts* opts,
                                bsp_spmm_plan** out);
/* A must have the pattern the plan was built for; values may differ. */
bsp_status bsp_spmm_execute(const bsp_spmm_plan* plan, const bsp_bsr_desc* A, const void* B,
                            int64_t ldb, void* C, int64_t ldc, void* stream);
bsp_status bsp_spmm_plan_destroy(bsp_spmm_plan* plan);

/* Multi-GPU row-panel SpMM with the all-gather fused into the kernel.  No
 * counterpart in the reference (it runs on one card).  Same as
 * bsp_spmm_execute, and every C element the kernel writes is also stored into
 * each of the n_peers (<= 7) other GPUs' C buffers, peer_C[i] pointing at the
 * element of the peer's C that corresponds to C[0][0] (same ldc), mapped into
 * this process over NVLink (bsp_ipc_import).  With A's block-rows split across
 * the GPUs, each GPU then ends with the whole C without a separate collective;
 * the caller synchronises the GPUs afterwards (any collective on the same
 * stream) before reading C.  DDA (row-stacked) plans only. */
bsp_status bsp_spmm_execute_replicated(const bsp_spmm_plan* plan, const bsp_bsr_desc* A, const void* B,
                                       int64_t ldb, void* C, int64_t ldc, void* const* peer_C,
                                       int32_t n_peers, void* stream);

/* CUDA IPC of device buffers between the processes of one node (one process
 * per GPU).  export: 64-byte handle of the allocation holding ptr, and ptr's
 * byte offset in it; import: map a peer's allocation, returns its base (add
 * the peer's offset); close: unmap. */
#define BSP_IPC_HANDLE_BYTES 64
bsp_status bsp_ipc_export(bsp_device* dev, const void* ptr, void* handle_out, int64_t* offset_out);
bsp_status bsp_ipc_import(bsp_device* dev, const void* handle, void** base_out);
bsp_status bsp_ipc_close(bsp_device* dev, void* base);
/* Plan facts: [0]=unit records (one per CTA of a pair for the CTA-pair
 * kernel) [1]=ctas [2]=entries per CTA [3]=n_tiles [4]=sub-row height
 * [5]=k chunk [6]=pipeline stages [7]=steps [8]=plan device bytes [9]=shared
 * memory per CTA [10]=TMEM columns [11]=kernel variant (0 swap-AB, 1 row-
 * stacked, 2 row-stacked on CTA pairs, 3 twin units on CTA pairs) [12]=producer warps [15]=int32 words
 * per step-table entry. */
bsp_status bsp_spmm_plan_info(const bsp_spmm_plan* plan, int64_t info[16]);

/* One-shot: plan, execute on `stream`, synchronise, destroy. */
bsp_status bsp_spmm(bsp_device* dev, const bsp_bsr_desc* A, const void* B, int64_t ldb, void* C,
                    int64_t ldc, bsp_dtype c_type, int64_t N, bsp_strategy strategy,
                    const bsp_spmm_opts* opts, void* stream);

/* Host-buffer entry point, the semantics of the reference planners: host
 * arrays in, host C out (M x N bf16, row-major, fully written).  Copies in,
 * plans, runs, copies out, synchronises (block_spmm/inc/host_code/
 * bsr_spmm_multicore_load_balanced_new_DM.cpp:502-535).  Device buffers come
 * from a grow-only workspace held by `dev`. */
bsp_status bsp_spmm_host(bsp_device* dev, int64_t M, int64_t K, int32_t R, int32_t C, int64_t nnzb,
                         const int32_t* row_ptr, const int32_t* col_idx, const uint16_t* values,
                         const uint16_t* B, int64_t N, uint16_t* C_out, bsp_strategy strategy,
                         const bsp_spmm_opts* opts);

/* bsp_spmm_host plus timing: after the first launch, `iters` more launches are
 * timed with CUDA events; *ms_per_launch = their mean device time.  This is the
 * is_profiling mode of the reference planners (1 + 10 EnqueueProgram calls,
 * block_spmm/inc/host_code/bsr_spmm_multicore_load_balanced_new_DM.cpp:507-513). */
bsp_status bsp_spmm_host_profile(bsp_device* dev, int64_t M, int64_t K, int32_t R, int32_t C,
                                 int64_t nnzb, const int32_t* row_ptr, const int32_t* col_idx,
                                 const uint16_t* values, const uint16_t* B, int64_t N,
                                 uint16_t* C_out, bsp_strategy strategy, const bsp_spmm_opts* opts,
                                 int32_t iters, double* ms_per_launch);

/* Several independent host-buffer SpMMs in one call (each job as
 * bsp_spmm_host: host arrays in, the whole of C_out written, bf16).  The
 * reference runs one product per host-code call and blocks on each
 * (block_spmm/inc/host_code/bsr_spmm_multicore_load_balanced_new_DM.cpp:
 * 499-535); here every job's inputs are queued on a copy stream first, the
 * plans are built on the host while they travel, and each job's kernel runs as
 * soon as its inputs have landed, so job k's C travels to the host while the
 * inputs of jobs k+1... still come in (PCIe copies in both directions at
 * once).  A job whose N is a multiple of 512 (and at least 1024) runs as two
 * column panels of one plan (four from N = 8192), with B and C copied panel
 * by panel.  Device
 * buffers for all jobs come from the device's grow-only workspace.  Returns
 * after every C_out is written. */
typedef struct bsp_spmm_host_job {
  int64_t M, K;          /* A is M x K with R x C blocks */
  int32_t R, C;
  int64_t nnzb;
  const int32_t* row_ptr;  /* host, M/R + 1 */
  const int32_t* col_idx;  /* host, nnzb */
  const uint16_t* values;  /* host, nnzb * R * C bf16 */
  const uint16_t* B;       /* host, K x N bf16, row-major */
  int64_t N;
  uint16_t* C_out;         /* host, M x N bf16, row-major */
} bsp_spmm_host_job;

bsp_status bsp_spmm_host_batch(bsp_device* dev, int32_t n_jobs, const bsp_spmm_host_job* jobs,
                               bsp_strategy strategy, const bsp_spmm_opts* opts);

/* SpMM that allocates no device memory.  No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc: code whose device memory is owned
 * up front by another allocator (a framework's caching allocator, a fixed
 * memory pool) or a process with a fixed memory budget.  It runs the same
 * Naive / SnF kernel as bsp_spmm_execute, but its scratch -- the work schedule
 * and the status word -- lives in a 4 MiB array inside libbsp.so's device
 * image, which every GPU that loads the library holds until the process exits.
 * The caller passes A (device arrays plus host copies of its pattern), B and C.
 *   - Schedules larger than the array (very large or very sparse-row-heavy
 *     patterns) are refused with BSP_ERR_UNSUPPORTED and a message.
 *   - All calls share the array; the previous call's contents stay in it, and
 *     each call rewrites the schedule and clears the status word.  Calls that
 *     overlap on the GPU (other streams or host threads on the same device)
 *     race on it.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current.
 *   - The call is synchronous: it waits for its stream and reads the status
 *     word back with a blocking copy, so it must not be called while any
 *     stream is capturing.  It reports kernel wait timeouts as
 *     BSP_ERR_TIMEOUT.
 *   - c_type BSP_BF16 or BSP_F32; A->values 16-byte aligned (as
 *     bsp_spmm_plan_create requires); BSP_ERR_INVALID_ARG otherwise.
 * strategy must be BSP_NAIVE or BSP_SNF.  The device is the current CUDA
 * device; no bsp_device is needed. */
bsp_status bsp_spmm_noalloc(const bsp_bsr_desc* A, const int32_t* host_row_ptr,
                            const int32_t* host_col_idx, const void* B, int64_t ldb, void* C,
                            int64_t ldc, int64_t N, bsp_dtype c_type, bsp_strategy strategy,
                            void* stream);

/* ---- SDDMM: out = mask (.) (A[M x K] * B[K x N]) on mask's pattern --------
 * Replaces SDDMMHostCodeFunctionPtr (block_sddmm/inc/host_code.hpp:104-115):
 * out_values[b*R*C + r*C + c] for every mask block b, in mask order; the output
 * pattern is the mask's pattern (bsr_sddmm_multicore_naive.cpp:333-346).
 * mask->values may be NULL: every mask value is 1 (pure sampling). */
typedef struct bsp_sddmm_plan bsp_sddmm_plan;

bsp_status bsp_sddmm_plan_create(bsp_device* dev, const bsp_bsr_desc* mask,
                                 const int32_t* host_row_ptr, const int32_t* host_col_idx,
                                 int64_t K, bsp_strategy strategy, const bsp_sddmm_opts* opts,
                                 bsp_sddmm_plan** out);
bsp_status bsp_sddmm_execute(const bsp_sddmm_plan* plan, const bsp_bsr_desc* mask, const void* A,
                             int64_t lda, const void* B, int64_t ldb, void* out_values,
                             void* stream);
bsp_status bsp_sddmm_plan_destroy(bsp_sddmm_plan* plan);
bsp_status bsp_sddmm_plan_info(const bsp_sddmm_plan* plan, int64_t info[16]);

bsp_status bsp_sddmm(bsp_device* dev, const bsp_bsr_desc* mask, const void* A, int64_t lda,
                     const void* B, int64_t ldb, int64_t K, void* out_values,
                     bsp_strategy strategy, const bsp_sddmm_opts* opts, void* stream);

/* Host-buffer SDDMM (reference semantics: host containers in, host BSR out
 * with the mask's pattern; bsr_sddmm_multicore_naive.cpp:6-352).
 * mask_values may be NULL (all ones). */
bsp_status bsp_sddmm_host(bsp_device* dev, int64_t M, int64_t N, int32_t R, int32_t C,
                          int64_t nnzb, const int32_t* row_ptr, const int32_t* col_idx,
                          const uint16_t* mask_values, const uint16_t* A, const uint16_t* B,
                          int64_t K, uint16_t* out_values, bsp_strategy strategy,
                          const bsp_sddmm_opts* opts);

/* bsp_sddmm_host plus timing of `iters` launches (see bsp_spmm_host_profile;
 * reference: block_sddmm/inc/host_code/bsr_sddmm_multicore_naive.cpp, is_profiling). */
bsp_status bsp_sddmm_host_profile(bsp_device* dev, int64_t M, int64_t N, int32_t R, int32_t C,
                                  int64_t nnzb, const int32_t* row_ptr, const int32_t* col_idx,
                                  const uint16_t* mask_values, const uint16_t* A,
                                  const uint16_t* B, int64_t K, uint16_t* out_values,
                                  bsp_strategy strategy, const bsp_sddmm_opts* opts, int32_t iters,
                                  double* ms_per_launch);

/* ---- SpGEMM: C_bsr = A_bsr[M x K] * B_bsr[K x N] -------------------------
 * Device form of bsr_matrix<T>::spgemm (sparse_common/bsr_matrix.hpp:741-810),
 * which the reference has only as a CPU golden: A has Ra x Ca blocks, B has
 * Ca x Cb blocks (the reference asserts W_A == H_B and C_A == R_B, 743-744),
 * C has Ra x Cb blocks.  C's pattern is every (i, j) with some A[i, k] and
 * B[k, j] stored, columns ascending per block-row (the reference's row-major
 * walk of its present[] map, 786-802); each block is accumulated in fp32 and
 * rounded to bf16 once.  Repeated column indices inside a row of A or B
 * contribute every stored block, as in the reference's loops.
 * Block sizes: Ra, Ca, Cb each 32, 64 or 128.
 * Options (bsp_spmm_opts): n_tiles 1 = 4 segments per unit (MMA N = 128),
 * 2 = 8 (N = 256), 0 = 8 unless 4 moves fewer operand bytes (sparse
 * products); steps_per_stage 1..4; producers; max_ctas; timeout_ms;
 * no_load_balance 0 = units dealt in order to the least-loaded CTA (default,
 * keeps neighbouring units concurrent for L2 reuse), 1 = contiguous split,
 * 2 = serpentine over units sorted by work.
 *
 * The plan holds C's pattern (computed on the host from A's and B's
 * patterns); read it with bsp_spgemm_pattern, allocate nnzb * Ra * Cb bf16
 * values, then execute. */
typedef struct bsp_spgemm_plan bsp_spgemm_plan;

bsp_status bsp_spgemm_plan_create(bsp_device* dev, const bsp_bsr_desc* A,
                                  const int32_t* a_host_row_ptr, const int32_t* a_host_col_idx,
                                  const bsp_bsr_desc* B, const int32_t* b_host_row_ptr,
                                  const int32_t* b_host_col_idx, const bsp_spmm_opts* opts,
                                  bsp_spgemm_plan** out);
/* C's pattern: *nnzb_out always; row_ptr_out[M/Ra + 1] and col_idx_out[nnzb]
 * (host arrays) when not NULL. */
bsp_status bsp_spgemm_pattern(const bsp_spgemm_plan* plan, int64_t* nnzb_out, int32_t* row_ptr_out,
                              int32_t* col_idx_out);
/* A->values, B->values: device bf16 blocks; out_values: device, nnzb*Ra*Cb. */
bsp_status bsp_spgemm_execute(const bsp_spgemm_plan* plan, const bsp_bsr_desc* A,
                              const bsp_bsr_desc* B, void* out_values, void* stream);
bsp_status bsp_spgemm_plan_destroy(bsp_spgemm_plan* plan);
/* info[0] units, [1] grid, [2] steps, [3] block products (A[i,k]*B[k,j] pairs),
 * [4] output blocks, [5] kc, [6] stages, [7] sub-steps per stage,
 * [8] table bytes, [9] shared memory, [10] TMEM columns, [11] segments per
 * unit, [12] producer warps, [13] TMA boxes over all steps (per k-chunk). */
bsp_status bsp_spgemm_plan_info(const bsp_spgemm_plan* plan, int64_t info[16]);

/* Host-buffer SpGEMM (bsr_matrix<T>::spgemm semantics: host BSR in, host BSR
 * out).  With out_values == NULL only *out_nnzb is written (size query);
 * otherwise out_row_ptr[M/Ra + 1], out_col_idx[out_cap], out_values[out_cap *
 * Ra * Cb] receive C and out_cap must be >= its block count.  iters > 0 also
 * times that many device launches (*ms_per_launch, may be NULL otherwise). */
bsp_status bsp_spgemm_host(bsp_device* dev, int64_t M, int64_t K, int64_t N, int32_t Ra, int32_t Ca,
                           int32_t Cb, int64_t a_nnzb, const int32_t* a_row_ptr,
                           const int32_t* a_col_idx, const uint16_t* a_values, int64_t b_nnzb,
                           const int32_t* b_row_ptr, const int32_t* b_col_idx,
                           const uint16_t* b_values, int64_t out_cap, int64_t* out_nnzb,
                           int32_t* out_row_ptr, int32_t* out_col_idx, uint16_t* out_values,
                           const bsp_spmm_opts* opts, int32_t iters, double* ms_per_launch);

/* ---- fused block-sparse attention step (one head) ------------------------
 * O = softmax_rows(scale * Q K^T on the mask's blocks) V: the chain of the
 * reference's SDDMM (block_sddmm/inc/host_code.hpp:104-115, golden
 * bsr_matrix::sddmm, sparse_common/bsr_matrix.hpp:816-857), a row softmax over
 * each row's stored positions, and its SpMM (block_spmm/inc/host_code.hpp:
 * 165-177, golden spmm_bfloat16, bsr_matrix.hpp:692-736), fused so that the
 * probabilities never reach DRAM.  The reference has no fused form (config 4
 * of its benchmark runs the two programs back to back).
 * mask: S x S pattern with 32 x 32 blocks (values ignored; a column repeated
 * in a row counts once).  Q, K, V: [S, d] row-major bf16 with leading
 * dimensions ldq, ldk, ldv (K is not transposed), d = 64 or 128.  O: [S, d]
 * bf16, ldo; rows of block-rows without mask blocks are written as 0.
 * Softmax in fp32 with exp2 of scale * log2(e) * S; P is rounded to bf16 for
 * the P V product; O is accumulated in fp32 and rounded once. */
typedef struct bsp_attn_plan bsp_attn_plan;

bsp_status bsp_attn_plan_create(bsp_device* dev, const bsp_bsr_desc* mask, const int32_t* host_row_ptr,
                                const int32_t* host_col_idx, int64_t d, const bsp_spmm_opts* opts,
                                bsp_attn_plan** out);
bsp_status bsp_attn_execute(const bsp_attn_plan* plan, const void* Q, int64_t ldq, const void* K,
                            int64_t ldk, const void* V, int64_t ldv, float scale, void* O,
                            int64_t ldo, void* stream);
bsp_status bsp_attn_plan_destroy(bsp_attn_plan* plan);
/* info[0] work units (parts of split units counted), [1] grid, [2] chunks,
 * [3] mask blocks (distinct), [4] S, [5] d, [6] parts of split units,
 * [7] split units, [8] table bytes, [9] shared memory, [10] TMEM columns.
 * Work units are 128 query rows.  When there are fewer units than CTAs, the
 * longest units are split into parts (consecutive key chunks, up to 16 per
 * unit) that run on the otherwise idle CTAs and are merged by the part that
 * finishes last; a plan therefore executes on one stream at a time.
 * Options: max_ctas; timeout_ms; n_tiles > 0 = instead cut every unit longer
 * than 5/4 n_tiles chunks into parts of about n_tiles chunks; group_rows = -1
 * never splits. */
bsp_status bsp_attn_plan_info(const bsp_attn_plan* plan, int64_t info[16]);

/* Host-buffer form: mask pattern, Q, K, V, O all host arrays ([S, d] dense). */
bsp_status bsp_attn_host(bsp_device* dev, int64_t S, int64_t d, int64_t nnzb, const int32_t* row_ptr,
                         const int32_t* col_idx, const uint16_t* Q, const uint16_t* K,
                         const uint16_t* V, float scale, uint16_t* O, const bsp_spmm_opts* opts);

/* ---- multi-GPU helpers (host logic; the exchange itself is NCCL) --------
 * Contiguous block-row ranges for `parts` GPUs balanced by nonzero-block
 * count (a generalisation of the reference's serpentine balancer,
 * block_spmm/inc/host_code/bsr_spmm_multicore_load_balanced_new_DM.cpp:346-393,
 * to ranges, so that each GPU's C row-panel is contiguous for the all-gather).
 * A range weighs its blocks plus one per row; the ranges minimise the
 * heaviest one, and among such splits each range takes about its share of
 * the rest.  bounds[parts + 1]: GPU p owns block-rows [bounds[p], bounds[p+1]). */
bsp_status bsp_partition_rows(const int32_t* row_ptr, int64_t n_block_rows, int32_t parts,
                              int64_t* bounds);

/* The reference's serpentine balancer, exposed for tests: rows sorted by
 * work, heaviest first (`perm`), dealt to `parts` workers in zig-zag passes.
 * owner[k] / slot[k]: worker and position of perm[k].
 * (block_spmm/inc/host_code.hpp:225-235 + load_balanced_new_DM.cpp:346-393) */
bsp_status bsp_serpentine_assign(int64_t n, int32_t parts, int32_t* owner, int32_t* slot);

#ifdef __cplusplus
}
#endif
#endif /* BSP_H_ */
