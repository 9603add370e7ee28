/*
 * CPU oracle for the grouped GEMM hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * Nothing in the product (the CUDA library under grouped_gemm_gpu_kernel_b200/) links, loads or
 * calls this file. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * leg use it, and only as the checker or as the timed CPU baseline.
 *
 * It restates, in plain C, the reference's host algorithm for the path:
 *   - tile counting            reference src/grouped_gemm.cu:54-65   (ceil_div, tile_count_for_problem)
 *   - prepare_problem_set      reference src/grouped_gemm.cu:967-1022 (stable sort + tile prefix sum)
 *   - the per-element contract reference src/grouped_gemm.cu:460-481,603-622
 *         D = alpha * (A x B) + beta * C, with C read only when c != NULL and beta != 0
 *   - the reference's host GEMM reference tests/test_correctness.cu:85-102 (FP32, natural k order,
 *         always reads C) -- restated as oracle_gemm_f32_refloop for the "port" CPU baseline.
 * The accuracy reference is oracle_gemm_f64: FP16 inputs decoded exactly, products and sums in FP64
 * (oracle_gemm_f64_fmt also takes BF16 inputs, for the library's BF16 extension, and
 * oracle_gemm_f64_epilogue adds the library's fused bias and activation; C given as float holds
 * 16-bit C values exactly).
 *
 * Parity pin: tests/test_oracle.py checks every function here against the reference's own host
 * code compiled from its sources (oracle/Makefile -> oracle/_ref/libgg_ref.so) and against the
 * committed fixtures in tests/golden/ that were produced by that build.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- FP16 decode (IEEE 754 binary16 -> binary64, exact) ---------------------------------- */
static double half_bits_to_double(uint16_t h) {
  const int sign = (h >> 15) & 1;
  const int expo = (h >> 10) & 0x1f;
  const int frac = h & 0x3ff;
  double v;
  if (expo == 0) {
    v = ldexp((double)frac, -24); /* subnormal */
  } else if (expo == 31) {
    v = frac ? NAN : INFINITY;
  } else {
    v = ldexp((double)(frac + 1024), expo - 25);
  }
  return sign ? -v : v;
}

double oracle_half_to_double(uint16_t h) { return half_bits_to_double(h); }

/* BF16 is the top half of an IEEE binary32: the value is exact as a float. */
static double bf16_bits_to_double(uint16_t h) {
  const uint32_t w = (uint32_t)h << 16;
  float f;
  memcpy(&f, &w, sizeof f);
  return (double)f;
}

double oracle_bf16_to_double(uint16_t h) { return bf16_bits_to_double(h); }

/* ---- 8-bit float decode (exact), the library's GG_INPUT_E4M3 / GG_INPUT_E5M2 -------------------
 * E4M3: sign, 4 exponent bits (bias 7), 3 mantissa bits; no infinities, S.1111.111 is NaN;
 *       exponent 0 is subnormal, m * 2^-9.
 * E5M2: sign, 5 exponent bits (bias 15), 2 mantissa bits; exponent 31 is inf (m = 0) or NaN;
 *       exponent 0 is subnormal, m * 2^-16. */
static double e4m3_bits_to_double(uint8_t v) {
  const int e = (v >> 3) & 0xf, m = v & 7;
  double x;
  if (e == 15 && m == 7) x = NAN;
  else if (e == 0) x = ldexp((double)m, -9);
  else x = ldexp((double)(8 + m), e - 10);
  return (v & 0x80) ? -x : x;
}

static double e5m2_bits_to_double(uint8_t v) {
  const int e = (v >> 2) & 0x1f, m = v & 3;
  double x;
  if (e == 31) x = m ? NAN : INFINITY;
  else if (e == 0) x = ldexp((double)m, -16);
  else x = ldexp((double)(4 + m), e - 17);
  return (v & 0x80) ? -x : x;
}

/* fmt 2 = E4M3, 3 = E5M2 */
double oracle_fp8_to_double(uint8_t v, int fmt) { return fmt == 3 ? e5m2_bits_to_double(v) : e4m3_bits_to_double(v); }

/* Element i of an operand array in input format fmt (0 FP16, 1 BF16: 2 bytes; 2 E4M3, 3 E5M2: 1). */
static double decode_elem(const void* p, int64_t i, int fmt) {
  switch (fmt) {
    case 1: return bf16_bits_to_double(((const uint16_t*)p)[i]);
    case 2: return e4m3_bits_to_double(((const uint8_t*)p)[i]);
    case 3: return e5m2_bits_to_double(((const uint8_t*)p)[i]);
    default: return half_bits_to_double(((const uint16_t*)p)[i]);
  }
}

/* ---- tile counting: reference src/grouped_gemm.cu:54-65 ---------------------------------- */
static int ceil_div_int(int x, int y) { return (x + y - 1) / y; }

int oracle_tile_count(int m, int n, int cta_m, int cta_n) {
  if (m <= 0 || n <= 0) return 0;
  return ceil_div_int(m, cta_m) * ceil_div_int(n, cta_n);
}

/* ---- prepare_problem_set: reference src/grouped_gemm.cu:967-1022 --------------------------
 * Sort modes (reference include/grouped_gemm/grouped_gemm.cuh:11-16):
 *   0 none            identity permutation
 *   1 by K            K descending, ties -> m*n (int64) descending            (src:977-984)
 *   2 by tiles        tile count descending, ties -> the by-K comparator      (src:986-993)
 *   3 by tiles then K the same comparator as 2                                (src:1000-1005)
 * std::stable_sort is restated as a stable top-down merge sort: on a tie the element from the
 * left run is taken first, so equal keys keep their input order. */
typedef struct {
  const int* m;
  const int* n;
  const int* k;
  int cta_m;
  int cta_n;
  int mode;
} sort_ctx;

/* returns nonzero when problem lhs must come strictly before problem rhs */
static int before_by_k(const sort_ctx* c, int lhs, int rhs) {
  if (c->k[lhs] != c->k[rhs]) return c->k[lhs] > c->k[rhs];
  const int64_t la = (int64_t)c->m[lhs] * c->n[lhs];
  const int64_t ra = (int64_t)c->m[rhs] * c->n[rhs];
  return la > ra;
}

static int before(const sort_ctx* c, int lhs, int rhs) {
  if (c->mode == 1) return before_by_k(c, lhs, rhs);
  const int lt = oracle_tile_count(c->m[lhs], c->n[lhs], c->cta_m, c->cta_n);
  const int rt = oracle_tile_count(c->m[rhs], c->n[rhs], c->cta_m, c->cta_n);
  if (lt != rt) return lt > rt;
  return before_by_k(c, lhs, rhs);
}

static void merge_sort(const sort_ctx* c, int* v, int* tmp, int lo, int hi) {
  if (hi - lo < 2) return;
  const int mid = lo + (hi - lo) / 2;
  merge_sort(c, v, tmp, lo, mid);
  merge_sort(c, v, tmp, mid, hi);
  int i = lo, j = mid, o = lo;
  while (i < mid && j < hi) {
    /* take the right element only when it must come strictly before the left one */
    if (before(c, v[j], v[i])) tmp[o++] = v[j++];
    else tmp[o++] = v[i++];
  }
  while (i < mid) tmp[o++] = v[i++];
  while (j < hi) tmp[o++] = v[j++];
  memcpy(v + lo, tmp + lo, (size_t)(hi - lo) * sizeof(int));
}

/* perm[count] receives sorted_to_original; offsets[count+1] the tile prefix sum.
 * Returns total_tiles, or -1 on bad arguments. */
int oracle_prepare(const int* m, const int* n, const int* k, int count, int cta_m, int cta_n,
                   int mode, int* perm, int* offsets) {
  if (count < 0 || (count > 0 && (!m || !n || !k || !perm)) || !offsets || cta_m <= 0 || cta_n <= 0)
    return -1;
  for (int i = 0; i < count; ++i) perm[i] = i;
  if (mode == 1 || mode == 2 || mode == 3) {
    sort_ctx c = {m, n, k, cta_m, cta_n, mode};
    int* tmp = (int*)malloc((size_t)(count > 0 ? count : 1) * sizeof(int));
    if (!tmp) return -1;
    merge_sort(&c, perm, tmp, 0, count);
    free(tmp);
  }
  offsets[0] = 0;
  for (int s = 0; s < count; ++s) {
    const int o = perm[s];
    offsets[s + 1] = offsets[s] + oracle_tile_count(m[o], n[o], cta_m, cta_n);
  }
  return offsets[count];
}

/* ---- FP64 GEMM (the accuracy reference) --------------------------------------------------------
 * Computes, for the selected rows (rows == NULL -> all m rows, in order) and all n columns:
 *   d[r*ldd + j]     = alpha * sum_k A[row,k]*B[k,j] + beta * C[row,j]   (C only if c && beta != 0)
 *   scale[r*ldd + j] = |alpha| * sqrt(sum_k (A[row,k]*B[k,j])^2) + |beta * C[row,j]|
 * 'r' indexes the output rows (0..nrows-1), 'row' the problem row. 'scale' (nullable) is the
 * magnitude that the relative-error metric of the tests divides by when |d| is small. */
/* The library's activations (GG_ACT_*): 1 = ReLU, max(z, 0) with NaN -> 0; 2 = GELU, tanh form
 * 0.5 z (1 + tanh(sqrt(2/pi) (z + 0.044715 z^3))) (Hendrycks and Gimpel). act_lipschitz bounds
 * |act'|, so an error e in z becomes at most act_lipschitz * e in act(z). */
static double activate(double z, int act) {
  if (act == 1) return z > 0.0 ? z : 0.0;
  if (act == 2) return 0.5 * z * (1.0 + tanh(0.7978845608028654 * (z + 0.044715 * z * z * z)));
  return z;
}

static double act_lipschitz(int act) { return act == 2 ? 1.13 : 1.0; } /* max GELU' = 1.1289... */

/* As oracle_gemm_f64, with A and B in input format `fmt` (0 = FP16, 1 = BF16, 2 = E4M3, 3 = E5M2;
 * `a` and `b` point to 2-byte or 1-byte elements accordingly), and the
 * library's epilogue extensions: bias (nullable, one value per output column, bias[j] for column
 * j) added after alpha*acc + beta*C, then activation `act`:
 *   d     = act(alpha * acc + beta * C + bias[j])
 *   scale = act_lipschitz(act) * (|alpha| * sqrt(sum (a*b)^2) + |beta * C| + |bias[j]|) */
void oracle_gemm_f64_epilogue(int m, int n, int k, const void* a, int lda, const void* b, int ldb,
                              const float* c, int ldc, float alpha, float beta, const int* rows, int nrows,
                              double* d, int ldd, double* scale, int fmt, const float* bias, int act) {
  if (m <= 0 || n <= 0) return;
  if (!rows) nrows = m;
  const int read_c = (c != NULL) && (beta != 0.0f);
  double* acc = (double*)calloc((size_t)n, sizeof(double));
  double* sq = (double*)calloc((size_t)n, sizeof(double));
  double* brow = (double*)malloc((size_t)n * sizeof(double));
  if (!acc || !sq || !brow) { free(acc); free(sq); free(brow); return; }
  for (int r = 0; r < nrows; ++r) {
    const int row = rows ? rows[r] : r;
    memset(acc, 0, (size_t)n * sizeof(double));
    memset(sq, 0, (size_t)n * sizeof(double));
    for (int kk = 0; kk < k; ++kk) {
      const double av = decode_elem(a, (int64_t)row * lda + kk, fmt);
      for (int j = 0; j < n; ++j) brow[j] = decode_elem(b, (int64_t)kk * ldb + j, fmt);
      for (int j = 0; j < n; ++j) {
        const double p = av * brow[j];
        acc[j] += p;
        sq[j] += p * p;
      }
    }
    for (int j = 0; j < n; ++j) {
      const double cv = read_c ? (double)c[(int64_t)row * ldc + j] : 0.0;
      const double bv = bias ? (double)bias[j] : 0.0;
      d[(int64_t)r * ldd + j] = activate((double)alpha * acc[j] + (double)beta * cv + bv, act);
      if (scale)
        scale[(int64_t)r * ldd + j] =
            act_lipschitz(act) * (fabs((double)alpha) * sqrt(sq[j]) + fabs((double)beta * cv) + fabs(bv));
    }
  }
  free(acc);
  free(sq);
  free(brow);
}

void oracle_gemm_f64_fmt(int m, int n, int k, const uint16_t* a, int lda, const uint16_t* b, int ldb,
                         const float* c, int ldc, float alpha, float beta, const int* rows, int nrows,
                         double* d, int ldd, double* scale, int fmt) {
  oracle_gemm_f64_epilogue(m, n, k, a, lda, b, ldb, c, ldc, alpha, beta, rows, nrows, d, ldd, scale, fmt, NULL, 0);
}

void oracle_gemm_f64(int m, int n, int k, const uint16_t* a, int lda, const uint16_t* b, int ldb,
                     const float* c, int ldc, float alpha, float beta, const int* rows, int nrows,
                     double* d, int ldd, double* scale) {
  oracle_gemm_f64_fmt(m, n, k, a, lda, b, ldb, c, ldc, alpha, beta, rows, nrows, d, ldd, scale, 0);
}

/* ---- the reference's host GEMM, restated (tests/test_correctness.cu:85-102) ---------------
 * Single-threaded FP32: acc += a*b in natural k order, then alpha*acc + beta*c. Like the
 * reference test it always reads C. Built with -ffp-contract=off so no FMA is formed. */
void oracle_gemm_f32_refloop(int m, int n, int k, const uint16_t* a, int lda, const uint16_t* b,
                             int ldb, const float* c, int ldc, float alpha, float beta, float* d,
                             int ldd) {
  if (m <= 0 || n <= 0) return;
  for (int i = 0; i < m; ++i) {
    for (int j = 0; j < n; ++j) {
      float acc = 0.0f;
      for (int kk = 0; kk < k; ++kk) {
        const float av = (float)half_bits_to_double(a[(int64_t)i * lda + kk]);
        const float bv = (float)half_bits_to_double(b[(int64_t)kk * ldb + j]);
        acc += av * bv;
      }
      const float cv = c[(int64_t)i * ldc + j];
      d[(int64_t)i * ldd + j] = alpha * acc + beta * cv;
    }
  }
}
