// Clamped lower Cholesky A = L L^T of r x r matrices (r a multiple of 32, r <= 512), one thread-block cluster per
// matrix, 32 x 32 tiles.
//
// The arithmetic is that of candidates/cuk/chol.cu (every value from the same operations in the same order):
//   factor_diag (chol.cu:115-180): pivot fmax(a_cc, tau) (a NaN pivot becomes tau), rd = rsqrt(pivot),
//     l = a * rd below the diagonal and pivot * rd on it, a_ik -= l_i l_k as one fused multiply-add;
//     the tile inverse by forward substitution with four interleaved chains (chol.cu:151-168);
//   panel P = A[i, j] Linv[j]^T and the trailing update A[i, k] -= P_i P_k^T as FMA chains from zero.
// The schedule is also the reference's: CTA rank 0 updates and factors the next diagonal tile ahead (look-ahead),
// the other CTAs update the trailing tiles round-robin and store the panel column.  What changes for B200: the
// CTAs of one matrix form a cluster and meet at the hardware cluster barrier (barrier.cluster, release/acquire)
// instead of a software grid barrier that spins on a global counter, so nothing here can wait forever, and many
// matrices run at once, one cluster each.  The reciprocal square root is the deterministic det_rsqrt.
#include "kernels.h"

namespace spq {

constexpr int LDS = TB + 1;

struct CholSmem {
    float inv[TB][LDS];
    float a[TB][LDS];
    float b[TB][LDS];
    float p[TB][LDS];
    float q[TB][LDS];
    float rd[TB];
};

__device__ __forceinline__ int r0_() { return 2 * (threadIdx.x / 16); }
__device__ __forceinline__ int c0_() { return 2 * (threadIdx.x % 16); }

// acc[u][v] += sum_m X[r0+u][m] Y[c0+v][m], m in order (chol.cu:63-71)
__device__ __forceinline__ void mm22(float (*X)[LDS], float (*Y)[LDS], float acc[2][2]) {
    const int r0 = r0_(), c0 = c0_();
#pragma unroll 8
    for (int m = 0; m < TB; ++m) {
        const float x0 = X[r0][m], x1 = X[r0 + 1][m], y0 = Y[c0][m], y1 = Y[c0 + 1][m];
        acc[0][0] = __fmaf_rn(x0, y0, acc[0][0]);
        acc[0][1] = __fmaf_rn(x0, y1, acc[0][1]);
        acc[1][0] = __fmaf_rn(x1, y0, acc[1][0]);
        acc[1][1] = __fmaf_rn(x1, y1, acc[1][1]);
    }
}

// dst = src Linv^T (chol.cu:105-112)
__device__ __forceinline__ void panel(float (*dst)[LDS], float (*src)[LDS], float (*inv)[LDS]) {
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    mm22(src, inv, acc);
    const int r0 = r0_(), c0 = c0_();
    dst[r0][c0] = acc[0][0];
    dst[r0][c0 + 1] = acc[0][1];
    dst[r0 + 1][c0] = acc[1][0];
    dst[r0 + 1][c0 + 1] = acc[1][1];
}

// 32 x 32 tile load, all global loads issued before the shared stores (256 threads, 4 elements each)
__device__ __forceinline__ void load_tile(float (*dst)[LDS], const float* src, int ld) {
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int e = threadIdx.x + q * 256;
        v[q] = ldcg(src + (size_t)(e / TB) * ld + e % TB);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int e = threadIdx.x + q * 256;
        dst[e / TB][e % TB] = v[q];
    }
}

// factor the updated tile in S.a: write L[j, j] and Li[j]; S.inv <- the tile inverse (chol.cu:115-180)
__device__ void factor_diag(float* L, float* Li, int n, int j, float tau, CholSmem& S) {
    __syncthreads();
    if (threadIdx.x < 32) {
        const int i = threadIdx.x;
        float a[TB];
#pragma unroll
        for (int k = 0; k < TB; ++k) a[k] = S.a[i][k];
        float myrd = 0.0f;
#pragma unroll
        for (int c = 0; c < TB; ++c) {
            const float piv = fmaxf(__shfl_sync(0xffffffffu, a[c], c), tau);
            const float rd = det_rsqrt(piv);
            const float l = (i > c) ? __fmul_rn(a[c], rd) : ((i == c) ? __fmul_rn(piv, rd) : 0.0f);
            myrd = (i == c) ? rd : myrd;
            a[c] = l;
#pragma unroll
            for (int k = c + 1; k < TB; ++k) {
                const float lk = __shfl_sync(0xffffffffu, l, k);
                a[k] = __fmaf_rn(-((i >= k) ? l : 0.0f), lk, a[k]);
            }
        }
#pragma unroll
        for (int k = 0; k < TB; ++k) S.a[i][k] = (k <= i) ? a[k] : 0.0f;
        S.rd[i] = myrd;
    }
    __syncthreads();
    if (threadIdx.x < 32) {  // lane kk: column kk of the inverse by forward substitution
        const int kk = threadIdx.x;
        float x[TB];
#pragma unroll
        for (int i = 0; i < TB; ++i) {
            float acc0 = (i == kk) ? 1.0f : 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
#pragma unroll
            for (int m = 0; m + 3 < i; m += 4) {
                acc0 = __fmaf_rn(-S.a[i][m], x[m], acc0);
                acc1 = __fmaf_rn(-S.a[i][m + 1], x[m + 1], acc1);
                acc2 = __fmaf_rn(-S.a[i][m + 2], x[m + 2], acc2);
                acc3 = __fmaf_rn(-S.a[i][m + 3], x[m + 3], acc3);
            }
#pragma unroll
            for (int m = (i / 4) * 4; m < i; ++m) acc0 = __fmaf_rn(-S.a[i][m], x[m], acc0);
            x[i] = (i < kk) ? 0.0f : __fmul_rn(__fadd_rn(__fadd_rn(acc0, acc1), __fadd_rn(acc2, acc3)), S.rd[i]);
        }
#pragma unroll
        for (int i = 0; i < TB; ++i) S.inv[i][kk] = x[i];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < TB * TB; e += blockDim.x) {
        const int r = e / TB, c = e % TB;
        L[(size_t)(j + r) * n + j + c] = S.a[r][c];
        Li[(size_t)(j + r) * TB + c] = S.inv[r][c];
    }
    __syncthreads();
}

template <int C>
__device__ __forceinline__ void sync_matrix() {
    if constexpr (C > 1) {
        cluster_sync_all();
    } else {
        __syncthreads();
    }
}

template <int C>
__global__ void __launch_bounds__(256) k_chol(float* __restrict__ A_all, float* __restrict__ L_all,
                                              float* __restrict__ Li_all, int n, const double* __restrict__ rowsq,
                                              int nsq, const float* __restrict__ tau_ptr, PassScal* __restrict__ scal,
                                              int zero_upper) {
    __shared__ CholSmem S;
    __shared__ float s_tau, s_shift;
    const int rank = (C > 1) ? (int)(blockIdx.x % C) : 0;
    const int b = blockIdx.x / C;
    float* A = A_all + (size_t)b * n * n;
    float* L = L_all + (size_t)b * n * n;
    float* Li = Li_all + (size_t)b * n * TB;
    const int nb = n / TB;

    if (threadIdx.x == 0) {
        if (rowsq) {
            double tot = 0.0;
            for (int a = 0; a < nsq; ++a) tot = __dadd_rn(tot, rowsq[(size_t)b * n + a]);
            const float nrm = __double2float_rn(__dsqrt_rn(tot));
            s_shift = __fmul_rn(1e-7f, nrm);
            s_tau = __fadd_rn(__fmul_rn(1e-8f, nrm), 1e-30f);
            if (rank == 0 && scal) {
                scal[b].nrm = nrm;
                scal[b].shift = s_shift;
                scal[b].tau = s_tau;
            }
        } else {
            s_shift = 0.0f;
            s_tau = *tau_ptr;
        }
    }
    __syncthreads();
    const float tau = s_tau;
    if (rowsq && rank == 0)
        for (int i = threadIdx.x; i < n; i += blockDim.x) A[(size_t)i * n + i] = __fadd_rn(A[(size_t)i * n + i], s_shift);
    if (zero_upper) {
        int t = 0;
        for (int ib = 0; ib < nb; ++ib)
            for (int kb = ib + 1; kb < nb; ++kb, ++t) {
                if (t % C != rank) continue;
                for (int e = threadIdx.x; e < TB * TB; e += blockDim.x)
                    L[(size_t)(ib * TB + e / TB) * n + kb * TB + e % TB] = 0.0f;
            }
    }
    sync_matrix<C>();

    if (rank == 0) {
        load_tile(S.a, A, n);
        factor_diag(L, Li, n, 0, tau, S);
    }
    sync_matrix<C>();
    for (int jb = 0; jb + 1 < nb; ++jb) {
        const int j = jb * TB, j1 = j + TB;
        if (rank == 0) {
            // look-ahead: P = A[j1, j] Linv[j]^T -> L[j1, j]; A[j1, j1] -= P P^T; factor it (S.inv <- Linv[j1])
            load_tile(S.b, A + (size_t)j1 * n + j, n);
            load_tile(S.a, A + (size_t)j1 * n + j1, n);
            __syncthreads();
            panel(S.p, S.b, S.inv);
            __syncthreads();
            {
                float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
                mm22(S.p, S.p, acc);
                const int r0 = r0_(), c0 = c0_();
#pragma unroll
                for (int u = 0; u < 2; ++u)
#pragma unroll
                    for (int v = 0; v < 2; ++v) {
                        const int r = r0 + u, c = c0 + v;
                        S.a[r][c] = __fsub_rn(S.a[r][c], acc[u][v]);
                        L[(size_t)(j1 + r) * n + j + c] = S.p[r][c];
                    }
            }
            factor_diag(L, Li, n, j1, tau, S);
        }
        if (C == 1 || rank > 0) {
            const int W = (C > 1) ? C - 1 : 1, me = (C > 1) ? rank - 1 : 0;
            bool have_inv = false;
            int t = 0;
            for (int ib = jb + 1; ib < nb; ++ib) {
                for (int kb = jb + 1; kb <= ib; ++kb) {
                    if (ib == jb + 1 && kb == jb + 1) continue;
                    if (t++ % W != me) continue;
                    const int i = ib * TB, kc = kb * TB;
                    const int r0 = r0_(), c0 = c0_();
                    float cur[2][2];
#pragma unroll
                    for (int u = 0; u < 2; ++u)
#pragma unroll
                        for (int v = 0; v < 2; ++v) cur[u][v] = ldcg(A + (size_t)(i + r0 + u) * n + kc + c0 + v);
                    if (!have_inv) load_tile(S.inv, Li + (size_t)j * TB, TB);
                    load_tile(S.a, A + (size_t)i * n + j, n);
                    load_tile(S.b, A + (size_t)kc * n + j, n);
                    have_inv = true;
                    __syncthreads();
                    panel(S.p, S.a, S.inv);
                    panel(S.q, S.b, S.inv);
                    __syncthreads();
                    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
                    mm22(S.p, S.q, acc);
#pragma unroll
                    for (int u = 0; u < 2; ++u)
#pragma unroll
                        for (int v = 0; v < 2; ++v) {
                            const int r = r0 + u, c = c0 + v;
                            A[(size_t)(i + r) * n + kc + c] = __fsub_rn(cur[u][v], acc[u][v]);
                            if (kb == jb + 1) L[(size_t)(i + r) * n + j + c] = S.p[r][c];
                        }
                    __syncthreads();
                }
            }
            if (C == 1) {  // single CTA: restore Linv[j1] for the next look-ahead
                load_tile(S.inv, Li + (size_t)j1 * TB, TB);
                __syncthreads();
            }
        }
        sync_matrix<C>();
    }
}

// ---- n <= 256: one CTA per matrix, the whole lower triangle in shared memory ----
// The same operations in the same order as above (and as chol.cu), scheduled for one CTA of 16 warps: per step j the
// panel tiles P_i = A[i, j] Linv[j]^T are computed in parallel and written in place (they are L[i, j]); then warp 0
// updates the next diagonal tile A[j+1, j+1] -= P_{j+1} P_{j+1}^T and factors it (look-ahead), while warps 1-15 apply
// A[i, k] -= P_i P_k^T to the other trailing tiles.  No global memory between the load and the stores of L and Li.
__device__ __forceinline__ void tc_named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
constexpr int SM_NB = 8;                       // up to 8 x 8 tiles (n <= 256)
constexpr int SM_TILE = TB * LDS;              // floats per stored tile
constexpr int SM_NT = 512;

__device__ __forceinline__ int lt_index(int ib, int kb) { return ib * (ib + 1) / 2 + kb; }

// factor the tile T in place with one warp (lane = row), T <- L tile (zeros above the diagonal); inv <- its inverse;
// rd <- the pivots' reciprocal square roots (chol.cu:115-180, the operations of factor_diag)
__device__ void factor_warp(float (*T)[LDS], float (*inv)[LDS], float* rd, float tau) {
    const int i = threadIdx.x & 31;
    float a[TB];
#pragma unroll
    for (int k = 0; k < TB; ++k) a[k] = T[i][k];
    float myrd = 0.0f;
#pragma unroll
    for (int c = 0; c < TB; ++c) {
        const float piv = fmaxf(__shfl_sync(0xffffffffu, a[c], c), tau);
        const float r = det_rsqrt(piv);
        const float l = (i > c) ? __fmul_rn(a[c], r) : ((i == c) ? __fmul_rn(piv, r) : 0.0f);
        myrd = (i == c) ? r : myrd;
        a[c] = l;
#pragma unroll
        for (int k = c + 1; k < TB; ++k) {
            const float lk = __shfl_sync(0xffffffffu, l, k);
            a[k] = __fmaf_rn(-((i >= k) ? l : 0.0f), lk, a[k]);
        }
    }
#pragma unroll
    for (int k = 0; k < TB; ++k) T[i][k] = (k <= i) ? a[k] : 0.0f;
    rd[i] = myrd;
    __syncwarp();
    const int kk = i;   // lane kk: column kk of the inverse by forward substitution
    float x[TB];
#pragma unroll
    for (int r = 0; r < TB; ++r) {
        float acc0 = (r == kk) ? 1.0f : 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
#pragma unroll
        for (int m = 0; m + 3 < r; m += 4) {
            acc0 = __fmaf_rn(-T[r][m], x[m], acc0);
            acc1 = __fmaf_rn(-T[r][m + 1], x[m + 1], acc1);
            acc2 = __fmaf_rn(-T[r][m + 2], x[m + 2], acc2);
            acc3 = __fmaf_rn(-T[r][m + 3], x[m + 3], acc3);
        }
#pragma unroll
        for (int m = (r / 4) * 4; m < r; ++m) acc0 = __fmaf_rn(-T[r][m], x[m], acc0);
        x[r] = (r < kk) ? 0.0f : __fmul_rn(__fadd_rn(__fadd_rn(acc0, acc1), __fadd_rn(acc2, acc3)), rd[r]);
    }
#pragma unroll
    for (int r = 0; r < TB; ++r) inv[r][kk] = x[r];
    __syncwarp();
}

// acc[u][v] = sum_m X[r0+u][m] Y[c0+v][m] for a 4 x 4 block, FMA chains from zero, m in order (chol.cu:63-71)
__device__ __forceinline__ void mm44_at(const float (*X)[LDS], const float (*Y)[LDS], int r0, int c0, float acc[4][4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = 0.0f;
#pragma unroll 4
    for (int m = 0; m < TB; ++m) {
        float x[4], y[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = X[r0 + u][m];
#pragma unroll
        for (int v = 0; v < 4; ++v) y[v] = Y[c0 + v][m];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[u][v] = __fmaf_rn(x[u], y[v], acc[u][v]);
    }
}

__global__ void __launch_bounds__(SM_NT, 1) k_chol_smem(float* __restrict__ A_all, float* __restrict__ L_all,
                                                        float* __restrict__ Li_all, int n,
                                                        const double* __restrict__ rowsq, int nsq,
                                                        const float* __restrict__ tau_ptr, PassScal* __restrict__ scal,
                                                        int zero_upper) {
    extern __shared__ float sm_f[];
    float (*tiles)[TB][LDS] = reinterpret_cast<float (*)[TB][LDS]>(sm_f);
    const int nb = n / TB;
    float (*inv)[LDS] = reinterpret_cast<float (*)[LDS]>(sm_f + (size_t)lt_index(nb, 0) * SM_TILE);
    float* rd = sm_f + (size_t)(lt_index(nb, 0) + 1) * SM_TILE;
    float* misc = rd + TB;   // [0] tau, [1] shift
    const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5;
    const float* A = A_all + (size_t)b * n * n;
    float* L = L_all + (size_t)b * n * n;
    float* Li = Li_all + (size_t)b * n * TB;

    // the row sums of G^2 staged in shared memory (the inverse's space, free until the first factor), so that the
    // in-order fp64 sum below does not wait on one global load per term
    double* rs = reinterpret_cast<double*>(inv);
    if (rowsq && tid < nsq) rs[tid] = rowsq[(size_t)b * n + tid];
    // the lower tiles of A (row-major, float4 reads in batches of 6 per thread), upper tiles of L zeroed on request
    const int n4 = n / 4, total = n * n4;
    for (int e0 = tid; e0 < total; e0 += 6 * SM_NT) {
        float4 v[6];
#pragma unroll
        for (int q = 0; q < 6; ++q) {
            const int e = e0 + q * SM_NT;
            if (e < total) {
                const int r = e / n4, c = 4 * (e % n4);
                if (c / TB <= r / TB) v[q] = __ldcg(reinterpret_cast<const float4*>(A + (size_t)r * n + c));
            }
        }
#pragma unroll
        for (int q = 0; q < 6; ++q) {
            const int e = e0 + q * SM_NT;
            if (e < total) {
                const int r = e / n4, c = 4 * (e % n4);
                const int ib = r / TB, kb = c / TB;
                if (kb > ib) {
                    if (zero_upper) *reinterpret_cast<float4*>(L + (size_t)r * n + c) = make_float4(0.f, 0.f, 0.f, 0.f);
                } else {
                    float* t = &tiles[lt_index(ib, kb)][r % TB][c % TB];
                    t[0] = v[q].x; t[1] = v[q].y; t[2] = v[q].z; t[3] = v[q].w;
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        if (rowsq) {
            double tot = 0.0;
            for (int a = 0; a < nsq; ++a) tot = __dadd_rn(tot, rs[a]);
            const float nrm = __double2float_rn(__dsqrt_rn(tot));
            misc[1] = __fmul_rn(1e-7f, nrm);
            misc[0] = __fadd_rn(__fmul_rn(1e-8f, nrm), 1e-30f);
            if (scal) {
                scal[b].nrm = nrm;
                scal[b].shift = misc[1];
                scal[b].tau = misc[0];
            }
        } else {
            misc[1] = 0.0f;
            misc[0] = *tau_ptr;
        }
    }
    __syncthreads();
    const float tau = misc[0];
    if (rowsq && tid < n) {   // G_ii += 1e-7 ||G||_F (kcholqr.py:108)
        float* d = &tiles[lt_index(tid / TB, tid / TB)][tid % TB][tid % TB];
        *d = __fadd_rn(*d, misc[1]);
    }
    __syncthreads();
    if (warp == 0) factor_warp(tiles[lt_index(0, 0)], inv, rd, tau);
    __syncthreads();

    for (int jb = 0; jb < nb; ++jb) {
        // the diagonal tile jb and its inverse are final: store them
        for (int e = tid; e < TB * TB; e += SM_NT) {
            const int r = e / TB, c = e % TB;
            L[(size_t)(jb * TB + r) * n + jb * TB + c] = tiles[lt_index(jb, jb)][r][c];
            Li[(size_t)(jb * TB + r) * TB + c] = inv[r][c];
        }
        if (jb + 1 == nb) break;
        // panels P_i = A[i, jb] Linv^T, i > jb (64 blocks of 4 x 4 per tile): all computed, then written in place
        // (they are L[i, jb])
        const int np = nb - 1 - jb;
        float pv[4][4];
        const int ptask = tid, pib = jb + 1 + ptask / 64, pw = ptask % 64;
        const bool has_p = ptask < np * 64;
        if (has_p) mm44_at(tiles[lt_index(pib, jb)], inv, 4 * (pw / 8), 4 * (pw % 8), pv);
        __syncthreads();
        if (has_p) {
            const int r0 = 4 * (pw / 8), c0 = 4 * (pw % 8);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
#pragma unroll
                for (int v = 0; v < 4; ++v) tiles[lt_index(pib, jb)][r0 + u][c0 + v] = pv[u][v];
                *reinterpret_cast<float4*>(L + (size_t)(pib * TB + r0 + u) * n + jb * TB + c0) =
                    make_float4(pv[u][0], pv[u][1], pv[u][2], pv[u][3]);
            }
        }
        __syncthreads();
        const int j1 = jb + 1;
        if (warp < 4) {
            // look-ahead on warps 0-3: A[j1, j1] -= P_j1 P_j1^T (64 blocks of 4 x 4), then warp 0 factors it
            float (*T)[LDS] = tiles[lt_index(j1, j1)];
            const float (*P)[LDS] = tiles[lt_index(j1, jb)];
            for (int w = tid; w < 64; w += 128) {
                const int r0 = 4 * (w / 8), c0 = 4 * (w % 8);
                float acc[4][4];
                mm44_at(P, P, r0, c0, acc);
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int v = 0; v < 4; ++v) T[r0 + u][c0 + v] = __fsub_rn(T[r0 + u][c0 + v], acc[u][v]);
            }
            tc_named_sync(1, 128);
            if (warp == 0) factor_warp(T, inv, rd, tau);
        } else {
            // A[i, k] -= P_i P_k^T for j1 <= k <= i, except (j1, j1), on warps 4-15
            const int ntr = np * (np + 1) / 2 - 1;
            for (int t = tid - 128; t < ntr * 64; t += SM_NT - 128) {
                int x = t / 64 + 1;   // trailing tile index, skipping (j1, j1) = index 0
                int ii = 0;
                while (x > ii) {
                    x -= ii + 1;
                    ++ii;
                }
                const int ib = j1 + ii, kb = j1 + x, w = t % 64, r0 = 4 * (w / 8), c0 = 4 * (w % 8);
                float acc[4][4];
                mm44_at(tiles[lt_index(ib, jb)], tiles[lt_index(kb, jb)], r0, c0, acc);
                float (*T)[LDS] = tiles[lt_index(ib, kb)];
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int v = 0; v < 4; ++v) T[r0 + u][c0 + v] = __fsub_rn(T[r0 + u][c0 + v], acc[u][v]);
            }
        }
        __syncthreads();
    }
}

size_t chol_smem_bytes(int n) { return ((size_t)(n / TB) * (n / TB + 1) / 2 + 1) * SM_TILE * 4 + (TB + 2) * 4; }

template <int C>
static cudaError_t launch_chol_c(float* A, float* L, float* Li, int n, int B, const double* rowsq, int nsq,
                                 const float* tau_ptr, PassScal* scal, int zero_upper, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C * B);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    int na = 0;
    if (C > 1) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = C;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        na = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k_chol<C>, A, L, Li, n, rowsq, nsq, tau_ptr, scal, zero_upper);
}

// Cluster size: a lone matrix spreads its trailing updates over 8 SMs; batches use 2 (many clusters at once).
cudaError_t launch_chol(float* A, float* L, float* Li, int n, int B, const double* rowsq, int nsq,
                        const float* tau_ptr, PassScal* scal, int zero_upper, cudaStream_t st) {
    const int nb = n / TB;
    if (nb <= SM_NB) {   // the whole lower triangle fits in one CTA's shared memory
        const size_t smem = chol_smem_bytes(n);
        cudaError_t e = cudaFuncSetAttribute(k_chol_smem, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k_chol_smem<<<B, SM_NT, smem, st>>>(A, L, Li, n, rowsq, nsq, tau_ptr, scal, zero_upper);
        return cudaGetLastError();
    }
    int C = (B >= 32) ? 2 : 8;
    if (nb <= 2) C = 1;
    else if (nb <= 4 && C > 2) C = 2;
    cudaError_t e;
    switch (C) {
        case 1: e = launch_chol_c<1>(A, L, Li, n, B, rowsq, nsq, tau_ptr, scal, zero_upper, st); break;
        case 2: e = launch_chol_c<2>(A, L, Li, n, B, rowsq, nsq, tau_ptr, scal, zero_upper, st); break;
        default: e = launch_chol_c<8>(A, L, Li, n, B, rowsq, nsq, tau_ptr, scal, zero_upper, st); break;
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace spq
