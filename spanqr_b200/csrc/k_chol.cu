// Clamped lower Cholesky A = L L^T of r x r matrices (r a multiple of 32, r <= 512) in 32 x 32 tiles: one
// thread-block cluster of C CTAs per matrix, the lower tiles held in the cluster's distributed shared memory.
//
// Arithmetic.  Every value is produced by the operations of the reference's kernel (candidates/cuk/chol.cu), in the
// same order, so L and the diagonal-tile inverses equal the CPU oracle's bit for bit:
//   diagonal tile (chol.cu:115-180): per column c, pivot fmax(a_cc, tau) (a NaN pivot becomes tau), rd = rsqrt(pivot)
//     (the deterministic det_rsqrt), l = a * rd below the diagonal and pivot * rd on it, a_ik -= l_i l_k as one fused
//     multiply-add; the tile's inverse by forward substitution with four interleaved chains (chol.cu:151-168);
//   panel P_i = A[i, j] Linv_j^T and trailing update A[i, k] -= P_i P_k^T, each product an FMA chain from zero over
//     m = 0..31 in order (chol.cu:63-71, 105-112, 244-258).
//
// Schedule (this file's own).  Block row i (tiles (i, 0..i)) lives in the shared memory of CTA i % C of the cluster.
// Step j of the factorisation:
//   1. cluster barrier: the inverse Linv_j (factored by the owner of row j) and every earlier update are complete;
//   2. every CTA copies Linv_j from its owner's shared memory (DSMEM) and computes the panels P_i of its own rows
//      i > j into its panel slots (they are also L[i, j], stored to global memory);
//   3. cluster barrier; every CTA copies the other CTAs' panels P_k (k > j) into its own panel slots;
//   4. the owner of row j + 1 updates tile (j + 1, j + 1) on two warps and factors it on one (look-ahead: Linv_{j+1}
//      is ready for the next step), while all other warps of the cluster apply A[i, k] -= P_i P_k^T to their tiles,
//      4 x 4 register blocks per thread.
// The barriers are hardware cluster barriers (barrier.cluster with release / acquire) reached the same number of times
// by every thread of the cluster, so nothing waits without end.  A lone matrix spreads over up to 8 SMs; batches use
// fewer CTAs per matrix and many clusters at once.  r > 256 needs C = 8 (the tiles of a 512 x 512 matrix do not fit
// the shared memory of fewer SMs).
#include "kernels.h"

namespace spq {

namespace {
constexpr int LDT = TB + 1;         // a stored tile row, padded: the column walks of the products are conflict-free
constexpr int TILE_F = TB * LDT;    // floats per stored tile
constexpr int NT = 384;             // 12 warps (no register spills in the unrolled diagonal factor)
constexpr int LA_THREADS = 128;     // look-ahead group (warps 0-3): panel, update and factor of the next diagonal tile
typedef float Tile[TB][LDT];

// CTA q of C owns block rows q, q + C, q + 2C, ... < nb; row i's tiles (i, 0..i) sit in consecutive slots
__host__ __device__ __forceinline__ int rows_of(int nb, int C, int q) { return q < nb ? (nb - 1 - q) / C + 1 : 0; }
__host__ __device__ __forceinline__ int tiles_of(int nb, int C, int q) {
    const int nr = rows_of(nb, C, q);
    return nr * (q + 1) + C * nr * (nr - 1) / 2;
}
// first slot of own row i (i = q + C t): rows q + C t' for t' < t hold q + C t' + 1 tiles each
__device__ __forceinline__ int row_slot(int C, int q, int i) {
    const int t = (i - q) / C;
    return t * (q + 1) + C * t * (t - 1) / 2;
}
__host__ __device__ __forceinline__ int max_tiles(int nb, int C) {
    int m = 0;
    for (int q = 0; q < C; ++q) m = tiles_of(nb, C, q) > m ? tiles_of(nb, C, q) : m;
    return m;
}
// own tiles, the panel slots (one per block row), this step's Linv_j, the inverses of the own diagonal tiles, the
// pivots' rsqrt, scalars
__host__ __device__ __forceinline__ size_t smem_floats(int nb, int C) {
    return (size_t)(max_tiles(nb, C) + nb + 1 + rows_of(nb, C, 0)) * TILE_F + TB + 4;
}

__device__ __forceinline__ int cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return (int)r;
}
// the generic address of the same shared-memory location in CTA `rank` of this cluster
template <typename T>
__device__ __forceinline__ const T* on_rank(const T* p, int rank) {
    uint64_t o;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(o) : "l"(p), "r"(rank));
    return reinterpret_cast<const T*>(o);
}
template <int C>
__device__ __forceinline__ void sync_cluster() {
    if constexpr (C > 1) cluster_sync_all();
    else __syncthreads();
}

// factor the tile T in place with one warp (lane = row), T <- L tile (zeros above the diagonal); inv <- its inverse;
// rd <- the pivots' reciprocal square roots (the operations of chol.cu:115-180).  Lane i's entries right of its
// diagonal are never read (lane i's l is 0 in the columns c > i, and they are zeroed at the end), so the update
// a_ik -= l_i l_k runs on every lane without the reference's select; and the next pivot, lane c + 1's updated
// diagonal, is computed from lane c + 1's own l (the same fused multiply-add) before the other lanes' l_{c+1} arrive,
// which keeps one shuffle off the column-to-column chain.
__device__ void factor_warp(float (*T)[LDT], float (*inv)[LDT], float* rd, float tau) {
    const int i = threadIdx.x & 31;
    float a[TB];
#pragma unroll
    for (int k = 0; k < TB; ++k) a[k] = T[i][k];
    float myrd = 0.0f;
    float pnext = a[0];   // lane c's diagonal entry, current before column c
#pragma unroll
    for (int c = 0; c < TB; ++c) {
        const float piv = fmaxf(__shfl_sync(0xffffffffu, pnext, c), tau);
        const float r = det_rsqrt(piv);
        const float l = (i > c) ? __fmul_rn(a[c], r) : ((i == c) ? __fmul_rn(piv, r) : 0.0f);
        myrd = (i == c) ? r : myrd;
        a[c] = l;
        if (c + 1 < TB) pnext = __fmaf_rn(-l, l, a[c + 1]);   // on lane c + 1: a_{c+1,c+1} - l_{c+1}^2
#pragma unroll
        for (int k = c + 1; k < TB; ++k) a[k] = __fmaf_rn(-l, __shfl_sync(0xffffffffu, l, k), a[k]);
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

// acc[u][v] = sum_m X[r0+u][m] Y[c0+v][m] for an RU x RV block, FMA chains from zero, m in order (chol.cu:63-71)
template <int RU, int RV>
__device__ __forceinline__ void mm_at(const float (*X)[LDT], const float (*Y)[LDT], int r0, int c0,
                                      float (&acc)[RU][RV]) {
#pragma unroll
    for (int u = 0; u < RU; ++u)
#pragma unroll
        for (int v = 0; v < RV; ++v) acc[u][v] = 0.0f;
#pragma unroll 4
    for (int m = 0; m < TB; ++m) {
        float x[RU], y[RV];
#pragma unroll
        for (int u = 0; u < RU; ++u) x[u] = X[r0 + u][m];
#pragma unroll
        for (int v = 0; v < RV; ++v) y[v] = Y[c0 + v][m];
#pragma unroll
        for (int u = 0; u < RU; ++u)
#pragma unroll
            for (int v = 0; v < RV; ++v) acc[u][v] = __fmaf_rn(x[u], y[v], acc[u][v]);
    }
}

// T -= acc on an RU x RV block
template <int RU, int RV>
__device__ __forceinline__ void sub_at(float (*T)[LDT], int r0, int c0, const float (&acc)[RU][RV]) {
#pragma unroll
    for (int u = 0; u < RU; ++u)
#pragma unroll
        for (int v = 0; v < RV; ++v) T[r0 + u][c0 + v] = __fsub_rn(T[r0 + u][c0 + v], acc[u][v]);
}

// a panel block into its panel slot
template <int RU>
__device__ __forceinline__ void put_panel(float (*slot)[LDT], int r0, int c0, const float (&acc)[RU][4]) {
#pragma unroll
    for (int u = 0; u < RU; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) slot[r0 + u][c0 + v] = acc[u][v];
}

// split phases of the cluster barrier (C = 1: of named barrier 2 over the CTA): arrive releases this thread's
// writes, wait acquires every arriving thread's
template <int C>
__device__ __forceinline__ void step_arrive() {
    if constexpr (C > 1) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    else asm volatile("bar.arrive 2, %0;" ::"n"(NT) : "memory");
}
template <int C>
__device__ __forceinline__ void step_arrive_wait() {
    if constexpr (C > 1)
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    else asm volatile("bar.sync 2, %0;" ::"n"(NT) : "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace

template <int C>
__global__ void __launch_bounds__(NT, 1) k_chol_dsm(float* __restrict__ A_all, float* __restrict__ L_all,
                                                    float* __restrict__ Li_all, int n, const double* __restrict__ rowsq,
                                                    int nsq, const float* __restrict__ tau_ptr,
                                                    PassScal* __restrict__ scal, int zero_upper) {
    extern __shared__ float4 smem4[];
    const int nb = n / TB;
    const int q = (C > 1) ? cta_rank() : 0;
    const int b = blockIdx.x / C;
    const int tid = threadIdx.x, warp = tid >> 5;
    Tile* T = reinterpret_cast<Tile*>(smem4);   // own tiles
    Tile* PB = T + max_tiles(nb, C);            // PB[i]: the panel P_i of the current step
    Tile& LINV = PB[nb];                        // this step's Linv_j
    Tile* IV = PB + nb + 1;                     // IV[t]: the inverse of own diagonal tile q + C t (read by the others)
    float* rd = &IV[rows_of(nb, C, 0)][0][0];
    float* misc = rd + TB;                      // [0] tau, [1] shift
    const float* A = A_all + (size_t)b * n * n;
    float* L = L_all + (size_t)b * n * n;
    float* Li = Li_all + (size_t)b * n * TB;
    const int nr = rows_of(nb, C, q);

    // the row sums of G^2 staged in shared memory (the panel slots are free until the first panel), so that the
    // in-order fp64 sum below does not wait on one global load per term
    double* rs = reinterpret_cast<double*>(&PB[0][0][0]);
    if (rowsq && tid < nsq) rs[tid] = rowsq[(size_t)b * n + tid];
    // own block rows of A (float4 reads, 4 in flight per thread)
    for (int t = 0; t < nr; ++t) {
        const int i = q + C * t, w4 = 8 * (i + 1), tot = TB * w4;   // float4s of row i's tiles
        Tile* Ti = T + row_slot(C, q, i);
        for (int e0 = tid; e0 < tot; e0 += 4 * NT) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = e0 + u * NT;
                if (e < tot)
                    v[u] = __ldcg(reinterpret_cast<const float4*>(A + (size_t)(i * TB + e / w4) * n + 4 * (e % w4)));
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = e0 + u * NT;
                if (e < tot) {
                    const int r = e / w4, c = 4 * (e % w4);
                    float* d = &Ti[c / TB][r][c % TB];
                    d[0] = v[u].x; d[1] = v[u].y; d[2] = v[u].z; d[3] = v[u].w;
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        if (rowsq) {   // kcholqr.py:107-109: nrm = ||G||_F, shift alpha nrm, tau 1e-8 nrm + 1e-30
            double tot = 0.0;
            for (int a = 0; a < nsq; ++a) tot = __dadd_rn(tot, rs[a]);
            const float nrm = __double2float_rn(__dsqrt_rn(tot));
            misc[1] = __fmul_rn(1e-7f, nrm);
            misc[0] = __fadd_rn(__fmul_rn(1e-8f, nrm), 1e-30f);
            if (scal && q == 0) {
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
    if (rowsq) {   // G_ii += alpha ||G||_F on this CTA's diagonal tiles (kcholqr.py:108)
        for (int e = tid; e < nr * TB; e += NT) {
            const int i = q + C * (e / TB), d = e % TB;
            float* g = &T[row_slot(C, q, i) + i][d][d];
            *g = __fadd_rn(*g, misc[1]);
        }
        __syncthreads();
    }
    if (q == 0 && warp == 0) factor_warp(T[0], IV[0], rd, tau);

    for (int j = 0; j < nb; ++j) {
        sync_cluster<C>();   // Linv_j is complete in its owner's IV slot; every update of step j - 1 is done
        if (j + 1 == nb) break;
        {   // Linv_j from its owner (slot j / C there)
            const float4* src = reinterpret_cast<const float4*>(&IV[j / C][0][0]);
            if (C > 1) src = on_rank(src, j % C);
            float4* dst = reinterpret_cast<float4*>(&LINV[0][0]);
            for (int e = tid; e < TILE_F / 4; e += NT) dst[e] = src[e];
        }
        __syncthreads();
        const int j1 = j + 1;
        const bool la = (j1 % C) == q;            // this CTA owns row j + 1
        const int t0 = (j + 1 - q + C - 1) / C;   // first own row index t with q + C t > j (on the la CTA, row j + 1)
        if (la && warp < LA_THREADS / 32) {
            // look-ahead group: P_{j+1} = A[j+1, j] Linv_j^T, released to the cluster at once; then tile (j+1, j+1)
            // -= P_{j+1} P_{j+1}^T and its factorisation, while the other warps of the cluster do the rest of the step
            const int r0 = 2 * (tid / 8), c0 = 4 * (tid % 8);
            const int s1 = row_slot(C, q, j1);
            float acc[2][4];
            mm_at<2, 4>(T[s1 + j], LINV, r0, c0, acc);
            put_panel<2>(PB[j1], r0, c0, acc);
            step_arrive<C>();
            named_sync(1, LA_THREADS);
            mm_at<2, 4>(PB[j1], PB[j1], r0, c0, acc);
            sub_at<2, 4>(T[s1 + j1], r0, c0, acc);
            named_sync(1, LA_THREADS);
            if (warp == 0) factor_warp(T[s1 + j1], IV[j1 / C], rd, tau);
            if (C > 1) cluster_wait();
        } else {
            const int nw = la ? NT - LA_THREADS : NT, wid = la ? tid - LA_THREADS : tid;
            // panels of this CTA's other rows i > j: P_i = A[i, j] Linv_j^T into PB[i], and to L[i, j]
            const int tp = la ? t0 + 1 : t0;
            for (int w = wid; w < (nr - tp) * 64; w += nw) {
                const int i = q + C * (tp + w / 64), r0 = 4 * ((w % 64) / 8), c0 = 4 * (w % 8);
                float acc[4][4];
                mm_at<4, 4>(T[row_slot(C, q, i) + j], LINV, r0, c0, acc);
                put_panel<4>(PB[i], r0, c0, acc);
            }
            step_arrive_wait<C>();   // every panel of step j is complete
            // the other CTAs' panels P_k (k > j) into this CTA's slots; this CTA's panels in place of A[i, j] (they
            // are L[i, j]; nothing reads column j again, and every global store of L waits until the end of the
            // kernel, so that no barrier's release has to wait for global writes)
            const int cnt = nb - 1 - j;
            for (int e = wid; e < cnt * (TILE_F / 4); e += nw) {
                const int k = j + 1 + e / (TILE_F / 4), f = e % (TILE_F / 4);
                float4* slot = reinterpret_cast<float4*>(&PB[k][0][0]) + f;
                if (k % C == q) reinterpret_cast<float4*>(&T[row_slot(C, q, k) + j][0][0])[f] = *slot;
                else if (C > 1) *slot = *on_rank(slot, k % C);
            }
            named_sync(3, nw);
            // A[i, k] -= P_i P_k^T for own rows i > j and j < k <= i, except (j + 1, j + 1) on the look-ahead CTA;
            // own rows from t0 on hold i - j trailing tiles each (k = j + 1 .. i), 64 4 x 4 blocks per tile
            int ntask = 0;
            for (int t = t0; t < nr; ++t) ntask += (q + C * t - j) * 64;
            for (int w = wid; w < ntask; w += nw) {
                int x = w / 64, t = t0;
                while (x >= q + C * t - j) {
                    x -= q + C * t - j;
                    ++t;
                }
                const int i = q + C * t, k = j + 1 + x;
                if (la && i == j1) continue;   // the look-ahead tile (k = j1 is the only trailing tile of row j1)
                const int r0 = 4 * ((w % 64) / 8), c0 = 4 * (w % 8);
                float acc[4][4];
                mm_at<4, 4>(PB[i], PB[k], r0, c0, acc);
                sub_at<4, 4>(T[row_slot(C, q, i) + k], r0, c0, acc);
            }
        }
    }
    // every tile of this CTA's block rows is final: L[i, 0..i], the inverse of tile (i, i), zeros right of it on request
    for (int t = 0; t < nr; ++t) {
        const int i = q + C * t, w4 = 8 * (i + 1), z4 = zero_upper ? (n - TB * (i + 1)) / 4 : 0;
        const Tile* Ti = T + row_slot(C, q, i);
        for (int e = tid; e < TB * (w4 + z4); e += NT) {
            const int r = e / (w4 + z4), c = 4 * (e % (w4 + z4));
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c < TB * (i + 1)) {
                const float* s = &Ti[c / TB][r][c % TB];
                v = make_float4(s[0], s[1], s[2], s[3]);
            }
            *reinterpret_cast<float4*>(L + (size_t)(i * TB + r) * n + c) = v;
        }
        for (int e = tid; e < TB * TB / 4; e += NT) {
            const int r = e / (TB / 4), c = 4 * (e % (TB / 4));
            const float* s = &IV[t][r][c];
            *reinterpret_cast<float4*>(Li + (size_t)(i * TB + r) * TB + c) = make_float4(s[0], s[1], s[2], s[3]);
        }
    }
}

size_t chol_smem_bytes(int n, int C) { return smem_floats(n / TB, C) * sizeof(float); }

namespace {
template <int C>
cudaError_t launch_c(float* A, float* L, float* Li, int n, int B, const double* rowsq, int nsq, const float* tau_ptr,
                     PassScal* scal, int zero_upper, cudaStream_t st) {
    const size_t smem = chol_smem_bytes(n, C);
    cudaError_t e = cudaFuncSetAttribute(k_chol_dsm<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C * B);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = C > 1 ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, k_chol_dsm<C>, A, L, Li, n, rowsq, nsq, tau_ptr, scal, zero_upper);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}
}  // namespace

// CTAs per matrix: 8 above r 256 (the tiles need the shared memory of 8 SMs).  Up to r 256 a batch of 16 or more
// matrices runs one CTA per matrix (the most work per SM; its parts run on concurrent streams, so the SMs are busy
// anyway: config 3's parts of 24 run 2.6% faster so than on clusters of 2), and a smaller batch (a lone matrix, a
// rank's share of a multi-GPU batch) spreads each matrix over up to 8 SMs (at most one per block row) while the whole
// batch stays within half of the SMs.  The bits do not depend on the cluster size.
int chol_cluster_size(int n, int B, int nsm) {
    const int nb = n / TB;
    if (nb > 8) return 8;
    if (B >= 16) return 1;
    int C = 1;
    while (C < 8 && 2 * C <= nb && (long long)B * 2 * C <= nsm / 2) C *= 2;
    return C;
}

cudaError_t launch_chol(float* A, float* L, float* Li, int n, int B, const double* rowsq, int nsq,
                        const float* tau_ptr, PassScal* scal, int zero_upper, cudaStream_t st) {
    if (n % TB || n < TB || n > MAX_R) return cudaErrorInvalidValue;
    int nsm = 0;
    const cudaError_t e = sm_count(&nsm);
    if (e != cudaSuccess) return e;
    switch (chol_cluster_size(n, B, nsm)) {
        case 1: return launch_c<1>(A, L, Li, n, B, rowsq, nsq, tau_ptr, scal, zero_upper, st);
        case 2: return launch_c<2>(A, L, Li, n, B, rowsq, nsq, tau_ptr, scal, zero_upper, st);
        case 4: return launch_c<4>(A, L, Li, n, B, rowsq, nsq, tau_ptr, scal, zero_upper, st);
        default: return launch_c<8>(A, L, Li, n, B, rowsq, nsq, tau_ptr, scal, zero_upper, st);
    }
}

}  // namespace spq
