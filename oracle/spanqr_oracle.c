/*
 * CPU ORACLE for spanqr's orth(X) -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the algorithm of the reference's GPU path
 *   orth.py:13-20 -> candidates/kcholqr.py:92-112 (kcholqr_f)
 * so that tests can check the CUDA product against it, and so that bench.py can time it as the CPU
 * baseline.  Nothing in the product (spanqr_b200/, libspanqr.so) links, loads or calls this file; only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
 *
 * Arithmetic is fp32 wherever the reference computes in fp32, fp64 where it sums in fp64, and every
 * fused multiply-add the reference's CUDA source contracts is written as an explicit fmaf (this file is
 * compiled with -ffp-contract=off, so no other contraction happens).  Where the reference's order is not
 * defined by its source (Triton tl.dot, cuBLAS SGEMM) a sequential order is used.
 *
 * Parity pins (tests/golden/make_golden.py): _pow2_scale, gram_f, gram_split, trsm_f and the whole of
 * kcholqr_f are checked against the reference's own Python/Triton code run on CPU (Triton interpreter);
 * the Cholesky restatement is checked against LAPACK on SPD inputs and against its clamping rules.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define TB 32

static int cdiv(int a, int b) { return (a + b - 1) / b; }
static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

/* ---------------------------------------------------------------------------------------------------
 * Reciprocal square root used by the clamped Cholesky.  The reference calls the hardware rsqrtf
 * (candidates/cuk/chol.cu:45), whose exact bits are not specified.  This build uses one deterministic
 * function that the CPU and the GPU evaluate with identical IEEE fp32 operations: the classic
 * integer-shift seed (Lomont's constant 0x5f375a86), two Newton-Raphson steps y <- y (1.5 - 0.5 x y^2)
 * and a last step on the residual computed with fused multiply-adds.  Within about one ulp for
 * normal x > 0 (checked against 1/sqrt in fp64 by the tests).
 * ------------------------------------------------------------------------------------------------- */
float oracle_rsqrt(float x) {
    uint32_t i;
    memcpy(&i, &x, 4);
    i = 0x5f375a86u - (i >> 1);
    float y;
    memcpy(&y, &i, 4);
    const float hx = 0.5f * x;
    for (int it = 0; it < 2; ++it) {
        float t = hx * y;
        t = t * y;
        t = 1.5f - t;
        y = y * t;
    }
    /* last step on the residual e = 1 - x y^2, with fused multiply-adds: y += (y/2) e */
    const float e = fmaf(-x, y * y, 1.0f);
    return fmaf(0.5f * y, e, y);
}

/* ---------------------------------------------------------------------------------------------------
 * kcholqr.py:29-30  _pow2_scale(m) = where(m > 0, exp2(-round(log2(clamp_min(m, 1e-38)))), 1)
 * As in the reference, log2 is rounded to fp32 first and round() is half-to-even on that fp32 value: near
 * 2^(k + 1/2) with large |k| the fp32 log2 is exactly k + 1/2 and the even neighbour wins.  The fp32 log2 is
 * the correctly rounded one (log2 in fp64, then rounded), which is what torch's CPU log2 returns there.
 * ------------------------------------------------------------------------------------------------- */
float oracle_pow2_scale(float m) {
    if (!(m > 0.0f)) return 1.0f;                 /* 0 and NaN */
    const float lo = 1e-38f;
    if (m < lo) m = lo;
    const float l2 = (float)log2((double)m);
    if (isinf(l2)) return 0.0f;                   /* exp2(-inf) */
    const float k = rintf(l2);                    /* half to even (default rounding mode) */
    return ldexpf(1.0f, -(int)k);
}

/* torch.linalg.vector_norm(X, ord=inf): max |x|, NaN-propagating (kcholqr.py:102) */
float oracle_absmax(const float* X, long long K, int r, long long ldx) {
    float m = 0.0f;
    int nan = 0;
    for (long long i = 0; i < K; ++i)
        for (int j = 0; j < r; ++j) {
            float a = fabsf(X[i * ldx + j]);
            if (a != a) nan = 1;
            else if (a > m) m = a;
        }
    return nan ? NAN : m;
}

/* ---------------------------------------------------------------------------------------------------
 * tri.py:329-378 gram_f / tri.py:262-298 gram_split: G = A^T A for A = s * Y.
 * Split count from the SM count (tri.py:365-370); within a split, Kahan over 32-row chunks whose dot is
 * an fp32 FMA chain; across splits an fp64 sum in split order, rounded to fp32 (tri.py:375).
 * ------------------------------------------------------------------------------------------------- */
static void gram_split_counts(int K, int n, int nsm, int* S_out, int* KS_out) {
    const int bt = 64, bk = 32;
    const int nt = cdiv(n, bt), up = nt * (nt + 1) / 2, tp = 3 * nsm;
    int S = imax(1, imin(cdiv(tp, up), cdiv(K, 4 * bk)));
    const int KS = cdiv(cdiv(K, S), bk) * bk;
    S = cdiv(K, KS);
    *S_out = S;
    *KS_out = KS;
}

/* column-major copy At[c][k] = s * Y[k][c] (s applied in fp32, as the kernel does on load) */
static float* transpose_scaled(const float* Y, int K, int n, long long ldy, float s, int has_s) {
    float* At = (float*)malloc(sizeof(float) * (size_t)K * n);
    for (int k = 0; k < K; ++k)
        for (int c = 0; c < n; ++c) {
            float v = Y[(long long)k * ldy + c];
            At[(size_t)c * K + k] = has_s ? v * s : v;
        }
    return At;
}

void oracle_gram_kahan(const float* Y, int K, int n, long long ldy, float s, int has_s, int nsm, float* G) {
    int S, KS;
    gram_split_counts(K, n, nsm, &S, &KS);
    float* At = transpose_scaled(Y, K, n, ldy, s, has_s);
#pragma omp parallel for schedule(dynamic, 1)
    for (int a = 0; a < n; ++a) {
        const float* xa = At + (size_t)a * K;
        for (int b = a; b < n; ++b) {
            const float* xb = At + (size_t)b * K;
            double tot = 0.0;
            float single = 0.0f;
            for (int sp = 0; sp < S; ++sp) {
                const int k0 = sp * KS, k1 = imin(k0 + KS, K);
                float acc = 0.0f, comp = 0.0f;
                for (int c0 = k0; c0 < k1; c0 += 32) {
                    const int c1 = imin(c0 + 32, k1);
                    float part = 0.0f;
                    for (int k = c0; k < c1; ++k) part = fmaf(xa[k], xb[k], part);
                    const float yv = part - comp;
                    const float t = acc + yv;
                    comp = (t - acc) - yv;
                    acc = t;
                }
                tot += (double)acc;
                single = acc;
            }
            const float g = (S > 1) ? (float)tot : single;
            G[(size_t)a * n + b] = g;
            G[(size_t)b * n + a] = g;
        }
    }
    free(At);
}

/* Y^T Y as a plain fp32 GEMM (kcholqr.py:106 and :20, cuBLAS SGEMM; its order is not specified):
 * FMA chains over 32-row chunks, chunk sums added in fp32 in order. */
void oracle_gram_plain(const float* Y, int K, int n, long long ldy, float* G) {
    float* At = transpose_scaled(Y, K, n, ldy, 1.0f, 0);
#pragma omp parallel for schedule(dynamic, 1)
    for (int a = 0; a < n; ++a) {
        const float* xa = At + (size_t)a * K;
        for (int b = a; b < n; ++b) {
            const float* xb = At + (size_t)b * K;
            float acc = 0.0f;
            for (int c0 = 0; c0 < K; c0 += 32) {
                const int c1 = imin(c0 + 32, K);
                float part = 0.0f;
                for (int k = c0; k < c1; ++k) part = fmaf(xa[k], xb[k], part);
                acc = acc + part;
            }
            G[(size_t)a * n + b] = acc;
            G[(size_t)b * n + a] = acc;
        }
    }
    free(At);
}

/* ---------------------------------------------------------------------------------------------------
 * candidates/cuk/chol.cu restated: lower Cholesky of A with pivots clamped at tau, 32 x 32 tiles.
 * Every value is produced by the same operations, in the same order, as the reference kernel:
 *   factor_diag (chol.cu:115-180): per column c, piv = fmax(a_cc, tau), rd = rsqrt(piv),
 *     l = a * rd below the diagonal, piv * rd on it, then a_ik -= l_i l_k (one FMA each);
 *     inverse of the tile by forward substitution with four interleaved chains (chol.cu:151-168);
 *   panel  P = A[i, j] Linv[j]^T  as FMA chains over m = 0..31 from zero (chol.cu:63-71, 105-112);
 *   update A[i, k] = A[i, k] - (P_i P_k^T), the product an FMA chain from zero (chol.cu:244-258).
 * The multi-CTA schedule of the reference does not change any of these values, so a sequential
 * walk over the tiles reproduces them.
 * A: n x n (lower tiles read, overwritten as workspace), L: n x n (upper part zeroed), Li: n x 32.
 * ------------------------------------------------------------------------------------------------- */
static void factor_diag(float* A, float* L, float* Li, int n, int j, float tau, float inv[TB][TB]) {
    float a[TB][TB];   /* a[i][k] = lane i's register row */
    float rd[TB];
    for (int i = 0; i < TB; ++i)
        for (int k = 0; k < TB; ++k) a[i][k] = A[(size_t)(j + i) * n + j + k];
    float myrd[TB];
    for (int i = 0; i < TB; ++i) myrd[i] = 0.0f;
    for (int c = 0; c < TB; ++c) {
        const float piv = fmaxf(a[c][c], tau);
        const float r = oracle_rsqrt(piv);
        float l[TB];
        for (int i = 0; i < TB; ++i) {
            l[i] = (i > c) ? a[i][c] * r : ((i == c) ? piv * r : 0.0f);
            if (i == c) myrd[i] = r;
        }
        for (int i = 0; i < TB; ++i) {
            a[i][c] = l[i];
            for (int k = c + 1; k < TB; ++k) {
                const float sel = (i >= k) ? l[i] : 0.0f;
                a[i][k] = fmaf(-sel, l[k], a[i][k]);
            }
        }
    }
    for (int i = 0; i < TB; ++i) {
        rd[i] = myrd[i];
        for (int k = 0; k < TB; ++k)
            if (k > i) a[i][k] = 0.0f;
    }
    for (int kk = 0; kk < TB; ++kk) {          /* column kk of the inverse */
        float x[TB];
        for (int i = 0; i < TB; ++i) {
            float acc0 = (i == kk) ? 1.0f : 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
            int m = 0;
            for (; m + 3 < i; m += 4) {
                acc0 = fmaf(-a[i][m], x[m], acc0);
                acc1 = fmaf(-a[i][m + 1], x[m + 1], acc1);
                acc2 = fmaf(-a[i][m + 2], x[m + 2], acc2);
                acc3 = fmaf(-a[i][m + 3], x[m + 3], acc3);
            }
            for (m = (i / 4) * 4; m < i; ++m) acc0 = fmaf(-a[i][m], x[m], acc0);
            x[i] = (i < kk) ? 0.0f : ((acc0 + acc1) + (acc2 + acc3)) * rd[i];
        }
        for (int i = 0; i < TB; ++i) inv[i][kk] = x[i];
    }
    for (int r = 0; r < TB; ++r)
        for (int c = 0; c < TB; ++c) {
            L[(size_t)(j + r) * n + j + c] = a[r][c];
            Li[(size_t)(j + r) * TB + c] = inv[r][c];
        }
}

/* dst[r][c] = sum_m src[r][m] inv[c][m] */
static void panel(float dst[TB][TB], const float* src, int ld, float inv[TB][TB]) {
    for (int r = 0; r < TB; ++r)
        for (int c = 0; c < TB; ++c) {
            float acc = 0.0f;
            for (int m = 0; m < TB; ++m) acc = fmaf(src[(size_t)r * ld + m], inv[c][m], acc);
            dst[r][c] = acc;
        }
}

int oracle_chol32(const float* G, int n, float tau, float* L, float* Li) {
    if (n <= 0 || n % TB) return 1;
    const int nb = n / TB;
    float* A = (float*)malloc(sizeof(float) * (size_t)n * n);
    memcpy(A, G, sizeof(float) * (size_t)n * n);
    memset(L, 0, sizeof(float) * (size_t)n * n);
    float (*inv)[TB][TB] = malloc(sizeof(float) * TB * TB * nb);
    factor_diag(A, L, Li, n, 0, tau, inv[0]);
    for (int jb = 0; jb + 1 < nb; ++jb) {
        const int j = jb * TB, j1 = j + TB;
        /* panels P_i = A[i, j] Linv[j]^T for every i > j (the same values every owner recomputes) */
        const int np = nb - jb - 1;
        float (*P)[TB][TB] = malloc(sizeof(float) * TB * TB * np);
#pragma omp parallel for
        for (int q = 0; q < np; ++q) panel(P[q], A + (size_t)(j1 + q * TB) * n + j, n, inv[jb]);
#pragma omp parallel for schedule(dynamic, 1)
        for (int q = 0; q < np; ++q) {
            const int ib = jb + 1 + q, i = ib * TB;
            for (int kb = jb + 1; kb <= ib; ++kb) {
                const int kc = kb * TB;
                float (*Pi)[TB] = P[q];
                float (*Pk)[TB] = P[kb - jb - 1];
                for (int r = 0; r < TB; ++r)
                    for (int c = 0; c < TB; ++c) {
                        float acc = 0.0f;
                        for (int m = 0; m < TB; ++m) acc = fmaf(Pi[r][m], Pk[c][m], acc);
                        float* a = A + (size_t)(i + r) * n + kc + c;
                        *a = *a - acc;
                    }
            }
            for (int r = 0; r < TB; ++r)
                for (int c = 0; c < TB; ++c) L[(size_t)(i + r) * n + j + c] = P[q][r][c];
        }
        free(P);
        factor_diag(A, L, Li, n, j1, tau, inv[jb + 1]);
    }
    free(inv);
    free(A);
    return 0;
}

/* ---------------------------------------------------------------------------------------------------
 * tri.py:384-412 trsm_f: Y = (s X + eps Z) L^-T, rows independent, 32-column blocks in order.
 * acc = s*x (+ eps*z); for each earlier block k: acc -= (Y_k L[j, k]^T) (dot as an FMA chain);
 * then Y_j = acc Li_j^T.  The reference's tf32x3 dots are fp32-accurate; fp32 chains stand in.
 * ------------------------------------------------------------------------------------------------- */
void oracle_trsm(const float* X, long long ldx, const float* Z, float s, int has_s, float eps, int has_z,
                 const float* L, const float* Li, int K, int n, float* Y, long long ldy) {
#pragma omp parallel for schedule(static)
    for (long long row = 0; row < K; ++row) {
        const float* x = X + row * ldx;
        const float* z = has_z ? Z + row * (long long)n : NULL;
        float* y = Y + row * ldy;
        for (int j = 0; j < n; j += TB) {
            float acc[TB];
            for (int c = 0; c < TB; ++c) {
                float v = x[j + c];
                if (has_s) v = v * s;
                if (has_z) v = v + eps * z[j + c];
                acc[c] = v;
            }
            for (int k = 0; k < j; k += TB)
                for (int c = 0; c < TB; ++c) {
                    const float* lrow = L + (size_t)(j + c) * n + k;
                    float d = 0.0f;
                    for (int m = 0; m < TB; ++m) d = fmaf(y[k + m], lrow[m], d);
                    acc[c] = acc[c] - d;
                }
            float out[TB];
            for (int c2 = 0; c2 < TB; ++c2) {
                const float* li = Li + (size_t)(j + c2) * TB;
                float d = 0.0f;
                for (int c = 0; c < TB; ++c) d = fmaf(acc[c], li[c], d);
                out[c2] = d;
            }
            for (int c = 0; c < TB; ++c) y[j + c] = out[c];
        }
    }
}

/* Frobenius norm (torch.linalg.matrix_norm, kcholqr.py:107): squares summed in fp64, one row at a time (columns
 * in order), then the row sums in order; rounded to fp32 after the square root. */
float oracle_fro(const float* G, int n) {
    double tot = 0.0;
    for (int a = 0; a < n; ++a) {
        double row = 0.0;
        for (int b = 0; b < n; ++b) {
            const double g = (double)G[(size_t)a * n + b];
            row += g * g;
        }
        tot += row;
    }
    return (float)sqrt(tot);
}

/* ---------------------------------------------------------------------------------------------------
 * kcholqr.py:16-23 _ns_mm: Newton-Schulz as a correction, Y <- Y + Y D with D = 0.5 (I - Y^T Y).
 * The reference takes step i < n-1's Gram from cuBLAS SGEMM (order unspecified) and the last step's from the
 * Kahan split Gram (gram_split, bt=64); here every step uses the split Gram (at least as accurate, fixed order).
 * D = eye.sub_(G).mul_(0.5) rounds twice; addmm(Y, Y, D) adds the fp32 product to Y.
 * ------------------------------------------------------------------------------------------------- */
void oracle_ns(float* Y, int K, int n, int steps, int nsm) {
    float* G = (float*)malloc(sizeof(float) * (size_t)n * n);
    float* D = (float*)malloc(sizeof(float) * (size_t)n * n);
    float* Dt = (float*)malloc(sizeof(float) * (size_t)n * n);
    for (int it = 0; it < steps; ++it) {
        oracle_gram_kahan(Y, K, n, n, 1.0f, 0, nsm, G);
        for (int a = 0; a < n; ++a)
            for (int b = 0; b < n; ++b) {
                const float e = (a == b) ? 1.0f : 0.0f;
                const float t = e - G[(size_t)a * n + b];
                D[(size_t)a * n + b] = t * 0.5f;
                Dt[(size_t)b * n + a] = t * 0.5f;
            }
#pragma omp parallel for schedule(static)
        for (long long row = 0; row < K; ++row) {
            float* y = Y + row * (long long)n;
            float tmp[1024];
            for (int b = 0; b < n; ++b) {
                const float* d = Dt + (size_t)b * n;
                float acc = 0.0f;
                for (int a = 0; a < n; ++a) acc = fmaf(y[a], d[a], acc);
                tmp[b] = y[b] + acc;
            }
            memcpy(y, tmp, sizeof(float) * n);
        }
    }
    free(G);
    free(D);
    free(Dt);
}

/* ---------------------------------------------------------------------------------------------------
 * kcholqr.py:92-112 kcholqr_f(X, eps=5e-7, alpha=1e-7, tau=1e-8, ns=2):
 *   s = pow2_scale(max|X|); 3 passes of {G = gram (pass 0: Kahan split Gram of s X, dust excluded;
 *   later: the reference's cuBLAS SGEMM, here the same split Gram), nrm = ||G||_F, G_ii += alpha nrm, (L, Li) = chol32(G, tau nrm + 1e-30),
 *   Y = trsm(Y, L, Li) with s X + eps Z on pass 0}; then _ns_mm(Y, ns).
 * Z: the dust, K x r, unit columns (kcholqr.py:83-89; the caller builds it).
 * Returns 0, or 1 for an unsupported shape (r % 32 != 0; the reference then falls back to Householder).
 * ------------------------------------------------------------------------------------------------- */
int oracle_kcholqr_f(const float* X, long long ldx, const float* Z, int K, int r, float eps, float alpha,
                     float tau_rel, int ns, int nsm, float* Q) {
    if (r <= 0 || r % TB || r > 1024 || K < r) return 1;
    const float m = oracle_absmax(X, K, r, ldx);
    const float s = oracle_pow2_scale(m);
    float* G = (float*)malloc(sizeof(float) * (size_t)r * r);
    float* L = (float*)malloc(sizeof(float) * (size_t)r * r);
    float* Li = (float*)malloc(sizeof(float) * (size_t)r * TB);
    float* Y = (float*)malloc(sizeof(float) * (size_t)K * r);
    for (int p = 0; p < 3; ++p) {
        if (p == 0) oracle_gram_kahan(X, K, r, ldx, s, 1, nsm, G);
        else oracle_gram_kahan(Y, K, r, r, 1.0f, 0, nsm, G);
        const float nrm = oracle_fro(G, r);
        const float shift = alpha * nrm;
        for (int i = 0; i < r; ++i) G[(size_t)i * r + i] = G[(size_t)i * r + i] + shift;
        const float tau = tau_rel * nrm + 1e-30f;
        oracle_chol32(G, r, tau, L, Li);
        if (p == 0) oracle_trsm(X, ldx, Z, s, 1, eps, 1, L, Li, K, r, Y, r);
        else oracle_trsm(Y, r, NULL, 1.0f, 0, 0.0f, 0, L, Li, K, r, Y, r);
    }
    oracle_ns(Y, K, r, ns, nsm);
    memcpy(Q, Y, sizeof(float) * (size_t)K * r);
    free(G);
    free(L);
    free(Li);
    free(Y);
    return 0;
}

/* orth(X) with the reference's constants (kcholqr.py:92) */
int oracle_orth(const float* X, long long ldx, const float* Z, int K, int r, int nsm, float* Q) {
    return oracle_kcholqr_f(X, ldx, Z, K, r, 5e-7f, 1e-7f, 1e-8f, 2, nsm, Q);
}

/* a batch of independent matrices, one per thread (the CPU baseline for orth_batched) */
int oracle_orth_batch(const float* const* X, const float* const* Z, const int* K, int r, int B, int nsm,
                      float* const* Q) {
    int bad = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(| : bad)
    for (int b = 0; b < B; ++b) {
        bad |= oracle_kcholqr_f(X[b], r, Z[b], K[b], r, 5e-7f, 1e-7f, 1e-8f, 2, nsm, Q[b]);
    }
    return bad;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
