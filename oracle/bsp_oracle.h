/* CPU restatement of the reference's golden block-sparse multiplies.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this library, and only as the checker.
 * The product library (libbsp.so) never links or calls it.
 *
 * Pinned against the reference's own golden (oracle/_ref, built from the
 * reference sources) and against the committed fixtures in tests/golden/.
 *
 * All bf16 values travel as raw uint16 bit patterns; bf16 -> f32 is exact and
 * f32 -> bf16 rounds to nearest even.
 */
#ifndef BSP_ORACLE_H
#define BSP_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint16_t bsp_oracle_f32_to_bf16(float f);
float bsp_oracle_bf16_to_f32(uint16_t b);

/* C[H x N] = A_bsr[H x W] * B[W x N], bf16 in/out, fp32 accumulate, block-rows
 * [row_begin, row_end) only (rows outside are not touched).  Follows
 * bsr_matrix::spmm_bfloat16, sparse_common/bsr_matrix.hpp:692-736. */
void bsp_oracle_spmm_bf16(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                          const int32_t* indices, const uint16_t* data, int64_t N,
                          const uint16_t* B, uint16_t* out, int64_t row_begin, int64_t row_end);

/* Same product in fp32 throughout (the float instantiation of
 * bsr_matrix::spmm, sparse_common/bsr_matrix.hpp:859-881).  `out` is
 * overwritten for the selected block-rows. */
void bsp_oracle_spmm_f32(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                         const int32_t* indices, const float* data, int64_t N, const float* B,
                         float* out, int64_t row_begin, int64_t row_end);

/* out_blocks = mask (.) (A[H x K] * B[K x W]) on the mask's pattern, bf16
 * in/out.  `mask_data` may be NULL (every mask value is 1).  Follows
 * bsr_matrix::sddmm, sparse_common/bsr_matrix.hpp:816-857. */
void bsp_oracle_sddmm_bf16(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                           const int32_t* indices, const uint16_t* mask_data, int64_t K,
                           const uint16_t* A, const uint16_t* B, uint16_t* out_blocks,
                           int64_t row_begin, int64_t row_end);

void bsp_oracle_sddmm_f32(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                          const int32_t* indices, const float* mask_data, int64_t K,
                          const float* A, const float* B, float* out_blocks, int64_t row_begin,
                          int64_t row_end);

/* Serpentine ("zig-zag") assignment of non-empty rows to `parts` workers,
 * given `perm` = row ids sorted by work, heaviest first.  Writes, for every
 * position k of `perm`, the worker that receives perm[k] into owner_of_pos[k]
 * and the order in which that worker receives it into slot_of_pos[k].
 * Follows block_spmm/inc/host_code/bsr_spmm_multicore_load_balanced_new_DM.cpp:346-393. */
void bsp_oracle_serpentine(int64_t n, int64_t parts, int32_t* owner_of_pos, int32_t* slot_of_pos);

/* SpGEMM (bsr_matrix.hpp:741-810): symbolic pattern of A*B (returns the block
 * count, fills out_rp[nbr_a+1] and, when non-null, out_ci), then the values. */
int64_t bsp_oracle_spgemm_symbolic(int64_t nbr_a, int64_t nbc_b, const int32_t* a_rp,
                                   const int32_t* a_ci, const int32_t* b_rp, const int32_t* b_ci,
                                   int32_t* out_rp, int32_t* out_ci);
void bsp_oracle_spgemm_bf16(int64_t nbr_a, int64_t Ra, int64_t Ca, int64_t Cb, const int32_t* a_rp,
                            const int32_t* a_ci, const uint16_t* a_vals, const int32_t* b_rp,
                            const int32_t* b_ci, const uint16_t* b_vals, const int32_t* out_rp,
                            const int32_t* out_ci, uint16_t* out_vals);

/* Threaded driver: runs bsp_oracle_spmm_bf16 / _sddmm_bf16 on `nthreads`
 * disjoint block-row ranges split by equal block counts. */
void bsp_oracle_spmm_bf16_mt(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                             const int32_t* indices, const uint16_t* data, int64_t N,
                             const uint16_t* B, uint16_t* out, int64_t row_begin, int64_t row_end,
                             int32_t nthreads);
void bsp_oracle_sddmm_bf16_mt(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                              const int32_t* indices, const uint16_t* mask_data, int64_t K,
                              const uint16_t* A, const uint16_t* B, uint16_t* out_blocks,
                              int64_t row_begin, int64_t row_end, int32_t nthreads);

/* The reference's value generators, which draw from the C library rand()
 * after srand(seed).  First n_unit values rand() / RAND_MAX in float (the block
 * data of test_random_hang / _v2, block_spmm/inc/test_suite.hpp:584-646), then
 * n_signed values of the RAND content kind, float(RAND_MAX / 2 - rand()) / 2048
 * (sparse_common/bsr_matrix.hpp:23-24 and 54-55): the dense operand of
 * make_frozen_case (block_spmm/inc/profiling_suite.hpp:69-91) is n_signed =
 * K * N such values after srand(42).  Either output may be NULL when its count
 * is 0.  Uses the process-wide rand() state (not thread-safe). */
void bsp_oracle_rand_fill(uint32_t seed, int64_t n_unit, float* unit_out, int64_t n_signed,
                          float* signed_out);

#ifdef __cplusplus
}
#endif
#endif
