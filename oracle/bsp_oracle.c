/* CPU restatement of the reference's golden block-sparse multiplies.
 *
 * TEST INFRASTRUCTURE ONLY (see bsp_oracle.h): the checker for the CUDA path,
 * never part of it.  Pinned against the reference's own golden compiled from
 * its sources (oracle/_ref) and against the fixtures in tests/golden/.
 *
 * The loops are reordered relative to the reference for cache efficiency, but
 * every output element sees exactly the same fp32 operations in the same
 * order, so results are bit-identical to the reference golden (compiled
 * without FMA contraction, as both are here).
 */
#include "bsp_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

uint16_t bsp_oracle_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float bsp_oracle_bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

enum { TILE = 32 }; /* bsr_matrix.hpp:22 TILE_SIZE */

/* bsr_matrix.hpp:692-736.  For each block-row i and 32-row slab r, an fp32
 * tile accumulator (the "DST register") collects, block by block in storage
 * order and 32-wide chunk by chunk of the block's C columns, the partial dot
 * product over that chunk (itself summed from zero in column order); the tile
 * is rounded to bf16 once at the end. */
void bsp_oracle_spmm_bf16(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                          const int32_t* indices, const uint16_t* data, int64_t N,
                          const uint16_t* B, uint16_t* out, int64_t row_begin, int64_t row_end) {
  (void)H;
  (void)W;
  float* tile = (float*)malloc(sizeof(float) * TILE * N);
  float* part = (float*)malloc(sizeof(float) * N);
  float* bf = (float*)malloc(sizeof(float) * TILE * N);
  for (int64_t i = row_begin; i < row_end; ++i) {
    for (int64_t r = 0; r < R; r += TILE) {
      const int64_t rmax = (r + TILE < R) ? r + TILE : R;
      memset(tile, 0, sizeof(float) * TILE * N);
      for (int64_t idx = indptr[i]; idx < indptr[i + 1]; ++idx) {
        const int64_t j = indices[idx];
        const uint16_t* a = data + idx * R * C;
        const uint16_t* b = B + j * C * N;
        for (int64_t c = 0; c < C; c += TILE) {
          const int64_t cmax = (c + TILE < C) ? c + TILE : C;
          /* widen this chunk of B once */
          for (int64_t cc = c; cc < cmax; ++cc)
            for (int64_t p = 0; p < N; ++p) bf[(cc - c) * N + p] = bsp_oracle_bf16_to_f32(b[cc * N + p]);
          for (int64_t rr = r; rr < rmax; ++rr) {
            for (int64_t p = 0; p < N; ++p) part[p] = 0.0f;
            for (int64_t cc = c; cc < cmax; ++cc) {
              const float av = bsp_oracle_bf16_to_f32(a[rr * C + cc]);
              const float* brow = bf + (cc - c) * N;
              for (int64_t p = 0; p < N; ++p) part[p] += av * brow[p];
            }
            float* trow = tile + (rr - r) * N;
            for (int64_t p = 0; p < N; ++p) trow[p] += part[p];
          }
        }
      }
      for (int64_t rr = r; rr < rmax; ++rr)
        for (int64_t p = 0; p < N; ++p)
          out[(i * R + rr) * N + p] = bsp_oracle_f32_to_bf16(tile[(rr - r) * N + p]);
    }
  }
  free(tile);
  free(part);
  free(bf);
}

/* bsr_matrix.hpp:859-881 (T = float): per block, per (r, p), a dot product
 * over the block's C columns summed from zero, added to the output element. */
void bsp_oracle_spmm_f32(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                         const int32_t* indices, const float* data, int64_t N, const float* B,
                         float* out, int64_t row_begin, int64_t row_end) {
  (void)H;
  (void)W;
  float* part = (float*)malloc(sizeof(float) * N);
  for (int64_t i = row_begin; i < row_end; ++i) {
    memset(out + i * R * N, 0, sizeof(float) * R * N);
    for (int64_t idx = indptr[i]; idx < indptr[i + 1]; ++idx) {
      const int64_t j = indices[idx];
      const float* a = data + idx * R * C;
      const float* b = B + j * C * N;
      for (int64_t r = 0; r < R; ++r) {
        for (int64_t p = 0; p < N; ++p) part[p] = 0.0f;
        for (int64_t c = 0; c < C; ++c) {
          const float av = a[r * C + c];
          for (int64_t p = 0; p < N; ++p) part[p] += av * b[c * N + p];
        }
        float* orow = out + (i * R + r) * N;
        for (int64_t p = 0; p < N; ++p) orow[p] += part[p];
      }
    }
  }
  free(part);
}

/* bsr_matrix.hpp:816-857: for every mask block (i, j) and element (r, c), an
 * fp32 dot product of row i*R+r of A with column j*C+c of B over all K,
 * multiplied by the mask value in fp32, rounded once.  The output keeps the
 * mask's pattern, so out_blocks is indexed exactly like the mask's data. */
void bsp_oracle_sddmm_bf16(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                           const int32_t* indices, const uint16_t* mask_data, int64_t K,
                           const uint16_t* A, const uint16_t* B, uint16_t* out_blocks,
                           int64_t row_begin, int64_t row_end) {
  (void)H;
  float* dot = (float*)malloc(sizeof(float) * C);
  for (int64_t i = row_begin; i < row_end; ++i) {
    for (int64_t idx = indptr[i]; idx < indptr[i + 1]; ++idx) {
      const int64_t j = indices[idx];
      for (int64_t r = 0; r < R; ++r) {
        const uint16_t* arow = A + (i * R + r) * K;
        for (int64_t c = 0; c < C; ++c) dot[c] = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
          const float av = bsp_oracle_bf16_to_f32(arow[k]);
          const uint16_t* brow = B + k * W + j * C;
          for (int64_t c = 0; c < C; ++c) dot[c] += av * bsp_oracle_bf16_to_f32(brow[c]);
        }
        for (int64_t c = 0; c < C; ++c) {
          const int64_t e = idx * R * C + r * C + c;
          const float m = mask_data ? bsp_oracle_bf16_to_f32(mask_data[e]) : 1.0f;
          out_blocks[e] = bsp_oracle_f32_to_bf16(m * dot[c]);
        }
      }
    }
  }
  free(dot);
}

void bsp_oracle_sddmm_f32(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                          const int32_t* indices, const float* mask_data, int64_t K,
                          const float* A, const float* B, float* out_blocks, int64_t row_begin,
                          int64_t row_end) {
  (void)H;
  float* dot = (float*)malloc(sizeof(float) * C);
  for (int64_t i = row_begin; i < row_end; ++i) {
    for (int64_t idx = indptr[i]; idx < indptr[i + 1]; ++idx) {
      const int64_t j = indices[idx];
      for (int64_t r = 0; r < R; ++r) {
        const float* arow = A + (i * R + r) * K;
        for (int64_t c = 0; c < C; ++c) dot[c] = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
          const float av = arow[k];
          const float* brow = B + k * W + j * C;
          for (int64_t c = 0; c < C; ++c) dot[c] += av * brow[c];
        }
        for (int64_t c = 0; c < C; ++c) {
          const int64_t e = idx * R * C + r * C + c;
          const float m = mask_data ? mask_data[e] : 1.0f;
          out_blocks[e] = m * dot[c];
        }
      }
    }
  }
  free(dot);
}

/* bsr_matrix.hpp:741-810, pattern part: block (i, j) of A*B exists when some
 * A[i, k] and B[k, j] both exist; each output row lists its columns in
 * ascending order (the reference walks a dense present[] map row-major). */
int64_t bsp_oracle_spgemm_symbolic(int64_t nbr_a, int64_t nbc_b, const int32_t* a_rp,
                                   const int32_t* a_ci, const int32_t* b_rp, const int32_t* b_ci,
                                   int32_t* out_rp, int32_t* out_ci) {
  uint8_t* seen = (uint8_t*)calloc((size_t)(nbc_b > 0 ? nbc_b : 1), 1);
  int64_t total = 0;
  out_rp[0] = 0;
  for (int64_t i = 0; i < nbr_a; ++i) {
    for (int32_t a = a_rp[i]; a < a_rp[i + 1]; ++a) {
      const int32_t k = a_ci[a];
      for (int32_t b = b_rp[k]; b < b_rp[k + 1]; ++b) seen[b_ci[b]] = 1;
    }
    for (int64_t j = 0; j < nbc_b; ++j) {
      if (!seen[j]) continue;
      if (out_ci) out_ci[total] = (int32_t)j;
      ++total;
      seen[j] = 0;
    }
    out_rp[i + 1] = (int32_t)total;
  }
  free(seen);
  return total;
}

/* bsr_matrix.hpp:741-810, values: for every pair (A[i, k], B[k, j]) in A's
 * storage order and then B's, each element (r, p) of the product block is an
 * fp32 sum over c from zero in column order, added to the fp32 accumulator of
 * output block (i, j) (started at zero); every block is rounded to bf16 once.
 * Ra x Ca blocks of A, Ca x Cb blocks of B, Ra x Cb blocks out. */
void bsp_oracle_spgemm_bf16(int64_t nbr_a, int64_t Ra, int64_t Ca, int64_t Cb, const int32_t* a_rp,
                            const int32_t* a_ci, const uint16_t* a_vals, const int32_t* b_rp,
                            const int32_t* b_ci, const uint16_t* b_vals, const int32_t* out_rp,
                            const int32_t* out_ci, uint16_t* out_vals) {
  const int64_t ob = Ra * Cb;
  float* acc = NULL;
  int64_t acc_cap = 0;
  for (int64_t i = 0; i < nbr_a; ++i) {
    const int32_t o0 = out_rp[i], no = out_rp[i + 1] - out_rp[i];
    if (no == 0) continue;
    if ((int64_t)no * ob > acc_cap) {
      acc_cap = (int64_t)no * ob;
      acc = (float*)realloc(acc, (size_t)acc_cap * sizeof(float));
    }
    memset(acc, 0, (size_t)no * ob * sizeof(float));
    for (int32_t a = a_rp[i]; a < a_rp[i + 1]; ++a) {
      const int32_t k = a_ci[a];
      const uint16_t* ab = a_vals + (int64_t)a * Ra * Ca;
      for (int32_t b = b_rp[k]; b < b_rp[k + 1]; ++b) {
        const int32_t j = b_ci[b];
        int32_t lo = 0, hi = no; /* slot of column j in output row i */
        while (lo < hi) {
          const int32_t mid = (lo + hi) / 2;
          if (out_ci[o0 + mid] < j) lo = mid + 1;
          else hi = mid;
        }
        float* dst = acc + (int64_t)lo * ob;
        const uint16_t* bb = b_vals + (int64_t)b * Ca * Cb;
        for (int64_t r = 0; r < Ra; ++r)
          for (int64_t p2 = 0; p2 < Cb; ++p2) {
            float sum = 0.0f;
            for (int64_t c = 0; c < Ca; ++c)
              sum += bsp_oracle_bf16_to_f32(ab[r * Ca + c]) * bsp_oracle_bf16_to_f32(bb[c * Cb + p2]);
            dst[r * Cb + p2] += sum;
          }
      }
    }
    for (int64_t e = 0; e < (int64_t)no * ob; ++e)
      out_vals[(int64_t)o0 * ob + e] = bsp_oracle_f32_to_bf16(acc[e]);
  }
  free(acc);
}

/* bsr_spmm_multicore_load_balanced_new_DM.cpp:371-393.  Pass `it` (from 1)
 * hands the next `parts` heaviest rows, front of `perm`, to workers 0..parts-1
 * in order, then the `parts` rows counted back from the end of `perm` to
 * workers parts-1..0, until every row is placed. */
void bsp_oracle_serpentine(int64_t n, int64_t parts, int32_t* owner_of_pos, int32_t* slot_of_pos) {
  int64_t assigned = 0, it = 1;
  int32_t* fill = (int32_t*)calloc((size_t)parts, sizeof(int32_t));
  while (assigned < n) {
    int64_t k = (parts < n - assigned) ? parts : n - assigned;
    int64_t sub = 0;
    for (int64_t w = 0; w < k; ++w) {
      if (assigned++ >= n) break;
      const int64_t pos = parts * (it - 1) + sub;
      owner_of_pos[pos] = (int32_t)w;
      slot_of_pos[pos] = fill[w]++;
      ++sub;
    }
    k = (parts < n - assigned) ? parts : n - assigned;
    sub = parts - k;
    for (int64_t w = parts; w > parts - k; --w) {
      if (assigned++ >= n) break;
      const int64_t pos = n - parts * it + sub;
      owner_of_pos[pos] = (int32_t)(w - 1);
      slot_of_pos[pos] = fill[w - 1]++;
      ++sub;
    }
    ++it;
  }
  free(fill);
}

/* ---- threaded drivers ---------------------------------------------------- */

typedef struct {
  int kind; /* 0 spmm, 1 sddmm */
  int64_t H, W, R, C, N, K;
  const int32_t *indptr, *indices;
  const uint16_t *data, *B, *A;
  uint16_t* out;
  int64_t r0, r1;
} job_t;

static void* run_job(void* p) {
  job_t* j = (job_t*)p;
  if (j->kind == 0)
    bsp_oracle_spmm_bf16(j->H, j->W, j->R, j->C, j->indptr, j->indices, j->data, j->N, j->B,
                         j->out, j->r0, j->r1);
  else
    bsp_oracle_sddmm_bf16(j->H, j->W, j->R, j->C, j->indptr, j->indices, j->data, j->K, j->A,
                          j->B, j->out, j->r0, j->r1);
  return NULL;
}

static void run_split(job_t base, int32_t nthreads) {
  if (nthreads < 1) nthreads = 1;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
  job_t* jobs = (job_t*)malloc(sizeof(job_t) * nthreads);
  const int64_t b0 = base.indptr[base.r0], b1 = base.indptr[base.r1];
  int64_t r = base.r0;
  for (int t = 0; t < nthreads; ++t) {
    jobs[t] = base;
    jobs[t].r0 = r;
    if (t == nthreads - 1) {
      r = base.r1;
    } else {
      const int64_t target = b0 + (b1 - b0) * (t + 1) / nthreads;
      while (r < base.r1 && base.indptr[r] < target) ++r;
    }
    jobs[t].r1 = r;
    pthread_create(&th[t], NULL, run_job, &jobs[t]);
  }
  for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
}

void bsp_oracle_spmm_bf16_mt(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                             const int32_t* indices, const uint16_t* data, int64_t N,
                             const uint16_t* B, uint16_t* out, int64_t row_begin, int64_t row_end,
                             int32_t nthreads) {
  job_t j = {0, H, W, R, C, N, 0, indptr, indices, data, B, NULL, out, row_begin, row_end};
  run_split(j, nthreads);
}

void bsp_oracle_sddmm_bf16_mt(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                              const int32_t* indices, const uint16_t* mask_data, int64_t K,
                              const uint16_t* A, const uint16_t* B, uint16_t* out_blocks,
                              int64_t row_begin, int64_t row_end, int32_t nthreads) {
  job_t j = {1, H, W, R, C, 0, K, indptr, indices, mask_data, B, A, out_blocks, row_begin, row_end};
  run_split(j, nthreads);
}

/* Restates the reference generators' draws (see bsp_oracle.h): one srand, then
 * the unit-interval draws, then the signed RAND draws, in that order. */
void bsp_oracle_rand_fill(uint32_t seed, int64_t n_unit, float* unit_out, int64_t n_signed,
                          float* signed_out) {
  srand(seed);
  for (int64_t i = 0; i < n_unit; ++i) unit_out[i] = (float)rand() / (float)RAND_MAX;
  for (int64_t i = 0; i < n_signed; ++i) signed_out[i] = (float)(RAND_MAX / 2 - rand()) / 2048.0f;
}
