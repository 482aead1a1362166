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
                                              const float* __restrict__ tau_ptr, PassScal* __restrict__ scal,
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
            for (int a = 0; a < n; ++a) tot = __dadd_rn(tot, rowsq[(size_t)b * n + a]);
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

template <int C>
static cudaError_t launch_chol_c(float* A, float* L, float* Li, int n, int B, const double* rowsq,
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
    return cudaLaunchKernelEx(&cfg, k_chol<C>, A, L, Li, n, rowsq, tau_ptr, scal, zero_upper);
}

// Cluster size: a lone matrix spreads its trailing updates over 8 SMs; batches use 2 (many clusters at once).
cudaError_t launch_chol(float* A, float* L, float* Li, int n, int B, const double* rowsq, const float* tau_ptr,
                        PassScal* scal, int zero_upper, cudaStream_t st) {
    const int nb = n / TB;
    int C = (B >= 32) ? 2 : 8;
    if (nb <= 2) C = 1;
    else if (nb <= 4 && C > 2) C = 2;
    cudaError_t e;
    switch (C) {
        case 1: e = launch_chol_c<1>(A, L, Li, n, B, rowsq, tau_ptr, scal, zero_upper, st); break;
        case 2: e = launch_chol_c<2>(A, L, Li, n, B, rowsq, tau_ptr, scal, zero_upper, st); break;
        default: e = launch_chol_c<8>(A, L, Li, n, B, rowsq, tau_ptr, scal, zero_upper, st); break;
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace spq
