/*
 * bsp_testing.h -- host-only inspection of the planners in libbsp.so.
 *
 * No counterpart in the reference (its planners run inline in each host-code
 * function).  These entry points run the SpMM / SDDMM planner on the host,
 * without a GPU, and return the schedule it would upload, so that its
 * invariants (every output tile written once, every block multiplied once per
 * tile, balanced CTA lists) can be tested on a CPU-only machine.
 */
#ifndef BSP_TESTING_H_
#define BSP_TESTING_H_
#include "bsp.h"

#ifdef __cplusplus
extern "C" {
#endif

/* info[16]: as bsp_spmm_plan_info.  With null output buffers only `info` is
 * filled (use it to size them): units_out[info[0] * 8] (row0, nrows, r_off,
 * n0, nt, step_begin, step_end, row_mask per unit, in CTA order),
 * cta_begin_out[info[1] + 1], steps_out[info[7] * (1 + info[2])]
 * (column, then the block index of each group row or -1).  For the
 * row-stacked kernel (info[11] == 1) stage_list_out[info[13] * 16] and
 * cta_stage_begin_out[info[1] + 1] receive the per-CTA stage descriptors. */
bsp_status bsp_spmm_plan_inspect(int64_t M, int64_t K, int32_t R, int32_t C, int64_t nnzb,
                                 const int32_t* row_ptr, const int32_t* col_idx, int64_t N,
                                 bsp_dtype c_type, bsp_strategy strategy,
                                 const bsp_spmm_opts* opts, int32_t sm_count, int32_t max_smem,
                                 int64_t info[16], int32_t* units_out, int32_t* cta_begin_out,
                                 int32_t* steps_out, int32_t* stage_list_out,
                                 int32_t* cta_stage_begin_out);

/* The SpMM planner's operand traffic (host only): traffic[0] A bytes and
 * traffic[2] A boxes, traffic[1] B bytes and traffic[3] B boxes that the
 * plan's kernel moves with TMA into shared memory (absent blocks excluded).
 * The counterpart of the reference's per-core in0 / in1 DRAM read counts
 * (block_spmm/scripts/count_dram_reads.py); info as bsp_spmm_plan_info. */
bsp_status bsp_spmm_plan_traffic(int64_t M, int64_t K, int32_t R, int32_t C, int64_t nnzb,
                                 const int32_t* row_ptr, const int32_t* col_idx, int64_t N,
                                 bsp_strategy strategy, const bsp_spmm_opts* opts, int32_t sm_count,
                                 int32_t max_smem, int64_t info[16], int64_t traffic[4]);

/* units_out[info[0] * info[12]]: info[11] == 0 (swap-AB kernel): 12 words per
 * unit (row, r_off, nseg, pad, blk[4], col[4]); info[11] == 1 (row-stacked
 * kernel): 44 words per unit (row0, nseg, pad[2], seg_col[8], blk[4][8]). */
/* Row-stacked SpMM plans: the stacking order of the block-rows (entry e of
 * the stack, a unit's row0 + g, is block-row rows_out[e]).  *n_out = 0 when
 * the plan stacks consecutive block-rows; rows_out may be NULL to query n. */
bsp_status bsp_spmm_plan_entry_rows(int64_t M, int64_t K, int32_t R, int32_t C, int64_t nnzb,
                                    const int32_t* row_ptr, const int32_t* col_idx, int64_t N,
                                    bsp_strategy strategy, const bsp_spmm_opts* opts, int32_t sm_count,
                                    int32_t max_smem, int32_t* rows_out, int64_t* n_out);

bsp_status bsp_sddmm_plan_inspect(int64_t M, int64_t N, int32_t R, int32_t C, int64_t nnzb,
                                  const int32_t* row_ptr, const int32_t* col_idx, int64_t K,
                                  bsp_strategy strategy, const bsp_sddmm_opts* opts,
                                  int32_t sm_count, int32_t max_smem, int64_t info[16],
                                  int32_t* units_out, int32_t* cta_begin_out);

/* SpGEMM planner (A: M x K with Ra x Ca blocks, B: K x N with Ca x Cb).
 * info[16] as bsp_spgemm_plan_info.  With null output buffers only `info` is
 * filled: out_row_ptr[M/Ra + 1], out_col_idx[info[4]] (C's pattern),
 * units_out[info[0] * 48] (step_begin, n_steps, n_ent, nseg, seg_x[8],
 * ent_r[4], out_blk[4][8] per unit, in CTA order), steps_out[info[2] * 16]
 * (per step: a_y[4] first A row of each entry box or -32*L for L zero slabs,
 * b_z[8] first B block of each segment box or -L for L zero segments, then
 * the meta bytes a_meta[4], b_meta[8], 4 pad bytes: bit 7 box present, bits
 * 0-2 first slot, bits 3-4 log2 slots, bits 5-6 32-column slice of B),
 * cta_begin_out[info[1] + 1]. */
bsp_status bsp_spgemm_plan_inspect(int64_t M, int64_t K, int64_t N, int32_t Ra, int32_t Ca,
                                   int32_t Cb, int64_t a_nnzb, const int32_t* a_row_ptr,
                                   const int32_t* a_col_idx, int64_t b_nnzb,
                                   const int32_t* b_row_ptr, const int32_t* b_col_idx,
                                   const bsp_spmm_opts* opts, int32_t sm_count, int32_t max_smem,
                                   int64_t info[16], int32_t* out_row_ptr, int32_t* out_col_idx,
                                   int32_t* units_out, int32_t* steps_out, int32_t* cta_begin_out);

/* Attention planner (S x S mask with 32 x 32 blocks, head size d).
 * info[16] as bsp_attn_plan_info; units_out[info[0] * 8] (row0, chunk_begin,
 * n_chunks, n_parts, part, slot0, counter, pad per unit or part, in CTA
 * order), chunks_out[info[2] * 8] (kb[4]:
 * key block of each slot or -1, bits: bit 4 q + s set when block-row q of the
 * unit holds slot s, pad[3]), cta_begin_out[info[1] + 1]. */
bsp_status bsp_attn_plan_inspect(int64_t S, int64_t d, int64_t nnzb, const int32_t* row_ptr,
                                 const int32_t* col_idx, const bsp_spmm_opts* opts, int32_t sm_count,
                                 int32_t max_smem, int64_t info[16], int32_t* units_out,
                                 int32_t* chunks_out, int32_t* cta_begin_out);

/* Device address and size of a row-stacked SpMM plan's split-K counters:
 * *counters points at two sets of *per_set int32 counters; the next launch
 * uses set *next_set and zeroes the other one before any of its waits.
 * (Tests overwrite the idle set to stand for counts that a launch which gave
 * up after a timeout left behind.)  *counters is NULL without split-K. */
bsp_status bsp_testing_spmm_counters(const bsp_spmm_plan* plan, void** counters, int64_t* per_set,
                                     int32_t* next_set);

/* Fault injection for the bounded-wait tests of row-stacked (single-CTA DDA)
 * plans: stage_plus_one = k + 1 makes CTA 0's producer leave its k-th pipeline
 * stage unissued on every later launch of `plan` (0 turns it off).  The MMA
 * warp's wait for that stage then runs out after the plan's timeout_ms, every
 * role drains its own copies and MMAs, TMEM is freed, and
 * bsp_device_synchronize reports BSP_ERR_TIMEOUT; the device stays usable.
 * No barrier is left unbounded and no memory access changes. */
bsp_status bsp_testing_spmm_drop_stage(bsp_spmm_plan* plan, int32_t stage_plus_one);

#ifdef __cplusplus
}
#endif
#endif /* BSP_TESTING_H_ */
