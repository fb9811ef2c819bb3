/*
 * vbsr_oracle.c — TEST INFRASTRUCTURE ONLY. CPU restatement of the reference's double-accumulating
 * reference SpMM, used as the parity checker by tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs. Nothing in the product library links or calls this code.
 *
 * Follows vbsr::cpu_reference (King-Clawthorne/VarBlockSpMM src/format/vbsr.cpp:167-201):
 *   for each block row, for each block of the row in order, for each local row r and RHS column n:
 *     sum = 0.0 (double); for each local column k: sum += double(a[r + k*h]) * b[col_off + k + n*K]
 *     C[row_off + r + n*M] += float(sum)      (float accumulation, block order)
 * (the loops are reordered for speed, each element's arithmetic unchanged; see run_rows)
 * The result is bit-identical to the reference for every element: each element's arithmetic is
 * the same sequence of double FMA-free multiply-adds and float additions. Rows are independent, so
 * a row-partitioned multi-threaded run is also bit-identical.
 *
 * Parity pinning: tests/test_oracle_golden.py checks this restatement bit for bit against
 * tests/golden/ fixtures produced by the reference's own generate() + cpu_reference() (script
 * tests/golden/make_golden.py, which runs the reference compiled by oracle/Makefile).
 *
 * Also computes the per-element bound S = sum_k |a_ik| |b_kj| (double) used by the tolerance
 * |C - C_ref| <= 1e-5 * S.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "vbsr_b200.h"

#if defined(__GNUC__)
/* The reference is compiled without FMA contraction of its double multiply-add (g++ -O2 on
 * x86-64 does not contract across a double product and sum unless -ffp-contract=fast and FMA
 * are both enabled); keep it that way here. */
#pragma GCC optimize("fp-contract=off")
#endif

typedef struct {
  const vbsr_host_matrix_view* v;
  const float* B;
  int rhs;
  int32_t r0, r1;     /* row range of the whole call */
  int32_t a, b;       /* this thread's rows          */
  int64_t ldc;        /* rows of the output panel    */
  int64_t row_base;   /* row_scalar_off[r0]          */
  float* C;           /* may be NULL                 */
  double* S;          /* may be NULL                 */
  const float* Ctest; /* compare mode: may be NULL   */
  double max_ratio, max_abs;
  int64_t bad;
} job_t;

/* Per element (r, n) the arithmetic is exactly the reference's: a double sum over the block's
 * columns k in order, then a float addition per block in block order. The loops are arranged so
 * that the RHS columns n (independent elements) are innermost and contiguous, which lets the
 * compiler vectorise across them without changing any element's sequence of operations: per block
 * the B slice is transposed once into bt[k][n], and sums[r][n] collects the block's double sums. */
#define ORACLE_MAX_H 64
#define ORACLE_MAX_RHS 64
#if defined(__GNUC__) && defined(__x86_64__)
__attribute__((target_clones("avx2", "default")))
#endif
static void block_sums(const float* av, int h, int w, int rhs, const float* bt, double* sums,
                       double* bound) {
  for (int k = 0; k < w; ++k) {
    const float* b = bt + k * rhs;
    for (int r = 0; r < h; ++r) {
      const double a = (double)av[(int64_t)k * h + r];
      double* s = sums + r * rhs;
      double* bd = bound + r * rhs;
      for (int n = 0; n < rhs; ++n) {
        const double prod = a * (double)b[n];
        s[n] = s[n] + prod;
        bd[n] = bd[n] + fabs(prod);
      }
    }
  }
}

static void run_rows(job_t* j) {
  const vbsr_host_matrix_view* v = j->v;
  const int64_t K = v->col_scalar_off[v->block_cols];
  const int rhs = j->rhs;
  float bt[ORACLE_MAX_H * ORACLE_MAX_RHS];
  double sums[ORACLE_MAX_H * ORACLE_MAX_RHS], bound[ORACLE_MAX_H * ORACLE_MAX_RHS];
  float acc[ORACLE_MAX_H * ORACLE_MAX_RHS];
  for (int32_t i = j->a; i < j->b; ++i) {
    const int h = v->row_size[i];
    const int64_t orow = v->row_scalar_off[i] - j->row_base;
    for (int e = 0; e < h * rhs; ++e) {
      acc[e] = 0.0f;
      bound[e] = 0.0;
    }
    for (int32_t blk = v->row_ptr[i]; blk < v->row_ptr[i + 1]; ++blk) {
      const int c = v->block_col[blk];
      const int w = v->col_size[c];
      const float* bcol = j->B + v->col_scalar_off[c];
      for (int k = 0; k < w; ++k)
        for (int n = 0; n < rhs; ++n) bt[k * rhs + n] = bcol[k + (int64_t)n * K];
      for (int e = 0; e < h * rhs; ++e) sums[e] = 0.0;
      block_sums(v->values + v->value_off[blk], h, w, rhs, bt, sums, bound);
      for (int e = 0; e < h * rhs; ++e) acc[e] = acc[e] + (float)sums[e];
    }
    for (int r = 0; r < h; ++r) {
      for (int n = 0; n < rhs; ++n) {
        const float a = acc[r * rhs + n];
        const double bnd = bound[r * rhs + n];
        const int64_t o = orow + r + (int64_t)n * j->ldc;
        if (j->C) j->C[o] = a;
        if (j->S) j->S[o] = bnd;
        if (j->Ctest) {
          const double err = fabs((double)j->Ctest[o] - (double)a);
          const double lim = 1e-5 * bnd;
          if (err > j->max_abs) j->max_abs = err;
          if (!(err <= lim)) {
            j->bad += 1;
            const double ratio = bnd > 0 ? err / lim : INFINITY;
            if (ratio > j->max_ratio || isnan(ratio)) j->max_ratio = isnan(ratio) ? INFINITY : ratio;
          } else if (bnd > 0 && err / lim > j->max_ratio) {
            j->max_ratio = err / lim;
          }
          if (!isfinite(j->Ctest[o])) { j->bad += 1; j->max_ratio = INFINITY; }
        }
      }
    }
  }
}

static void* thread_main(void* arg) {
  run_rows((job_t*)arg);
  return NULL;
}

static int run_parallel(job_t* base, int threads, double* max_ratio, double* max_abs, int64_t* bad) {
  const int32_t rows = base->r1 - base->r0;
  if (threads < 1) threads = 1;
  if (threads > rows) threads = rows > 0 ? rows : 1;
  job_t* jobs = (job_t*)calloc((size_t)threads, sizeof(job_t));
  pthread_t* tid = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  if (!jobs || !tid) { free(jobs); free(tid); return -1; }
  for (int t = 0; t < threads; ++t) {
    jobs[t] = *base;
    jobs[t].a = base->r0 + (int32_t)((int64_t)rows * t / threads);
    jobs[t].b = base->r0 + (int32_t)((int64_t)rows * (t + 1) / threads);
    if (threads > 1) pthread_create(&tid[t], NULL, thread_main, &jobs[t]);
  }
  if (threads == 1) run_rows(&jobs[0]);
  double mr = 0, ma = 0;
  int64_t nb = 0;
  for (int t = 0; t < threads; ++t) {
    if (threads > 1) pthread_join(tid[t], NULL);
    if (jobs[t].max_ratio > mr) mr = jobs[t].max_ratio;
    if (jobs[t].max_abs > ma) ma = jobs[t].max_abs;
    nb += jobs[t].bad;
  }
  if (max_ratio) *max_ratio = mr;
  if (max_abs) *max_abs = ma;
  if (bad) *bad = nb;
  free(jobs);
  free(tid);
  return 0;
}

static int setup(job_t* j, const vbsr_host_matrix_view* v, const float* B, int rhs, int32_t r0,
                 int32_t r1) {
  if (!v || !B || (!v->values && v->values_len) || r0 < 0 || r1 > v->block_rows || r0 > r1) return -1;
  if (rhs != 8 && rhs != 16 && rhs != 32 && rhs != 64) return -1;
  memset(j, 0, sizeof *j);
  j->v = v;
  j->B = B;
  j->rhs = rhs;
  j->r0 = r0;
  j->r1 = r1;
  j->row_base = v->row_scalar_off[r0];
  j->ldc = v->row_scalar_off[r1] - v->row_scalar_off[r0];
  return 0;
}

/* C (and optionally S) for block rows [r0, r1): column-major, ld = row_scalar_off[r1] -
 * row_scalar_off[r0]. B is the full K x rhs panel. Returns 0 on success. */
int vbsr_oracle_spmm(const vbsr_host_matrix_view* v, const float* B, int rhs, int32_t r0,
                     int32_t r1, float* C, double* S, int threads) {
  job_t j;
  if (setup(&j, v, B, rhs, r0, r1)) return -1;
  j.C = C;
  j.S = S;
  return run_parallel(&j, threads, NULL, NULL, NULL);
}

/* Compares Ctest (same layout as vbsr_oracle_spmm's C) with the oracle element-wise under
 * |Ctest - C_ref| <= 1e-5 * S. Reports the largest error/limit ratio, the largest absolute error
 * and the number of violating (or non-finite) elements. */
int vbsr_oracle_compare(const vbsr_host_matrix_view* v, const float* B, int rhs, int32_t r0,
                        int32_t r1, const float* Ctest, int threads, double* max_ratio,
                        double* max_abs, int64_t* bad) {
  job_t j;
  if (setup(&j, v, B, rhs, r0, r1) || !Ctest) return -1;
  j.Ctest = Ctest;
  return run_parallel(&j, threads, max_ratio, max_abs, bad);
}
