// Host-side launchers of the spanqr kernels (one translation unit per kernel family).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace spq {

// Source of a kernel's input matrix: the caller's X, or the in-progress Q (which holds Y between passes).
enum Src : int { SRC_X = 0, SRC_Q = 1 };

// Pointer source for a kernel: a device table of per-matrix pointers, or (when tab is null) one pair by value.
struct PtrArg {
    const MatPtr* tab;
    MatPtr one;
};

// The scale applied on load: pow2_scale(max |X|) from the absmax bits, an explicit device scalar per matrix, or 1.
struct ScaleArg {
    const uint32_t* maxbits;  // [B] or null
    const float* s;           // [B] or null
};

// Split-K plan of the Gram: 128 x 128 tiles of the upper triangle (or, with b0 > 0, of the band ti < b0 <= tj: the
// cross product of the first 128 b0 columns with the rest), splits of a fixed number of rows.
struct GramPlan {
    int nt;      // tiles per side, n / 128 rounded up
    int tiles;   // upper tiles nt (nt + 1) / 2, or b0 (nt - b0) in band mode
    int S;       // splits
    int KS;      // rows per split
    int b0;      // 0: the upper triangle; else the first tile column of the band
};

// tile t of a plan -> (ti, tj)
__device__ __forceinline__ void gram_tile_of(const GramPlan& gp, int t, int& ti, int& tj) {
    if (gp.b0 > 0) {
        const int w = gp.nt - gp.b0;
        ti = t / w;
        tj = gp.b0 + t % w;
    } else {
        upper_tile(t, gp.nt, ti, tj);
    }
}

// the set-up kernel of the strided entry points, k_setup_strided(tab, X, sX, Q, sQ, B, maxbits, status): the only
// kernel of an orth call that takes X and Q as arguments (every later one reads them from the table)
const void* setup_strided_kernel();
cudaError_t launch_setup_strided(MatPtr* tab, const float* X, long long sX, float* Q, long long sQ, int B,
                                 uint32_t* maxbits, int* status, cudaStream_t st);
cudaError_t launch_setup_array(MatPtr* tab, const float* const* dX, float* const* dQ, int B, uint32_t* maxbits,
                               int* status, cudaStream_t st);
// host arrays of pointers, passed by value to the set-up kernel in chunks
// device timeout self-test: one warp waits up to limit_ns on an mbarrier phase that completes only if `arrive`;
// a wait that runs out ORs SELFTEST_TIMEOUT into *status
constexpr int SELFTEST_TIMEOUT = 0x80;
cudaError_t launch_wait_selftest(int arrive, unsigned long long limit_ns, int* status, cudaStream_t st);
int setup_host_launches(int B);   // kernels launch_setup_host issues for B pointer pairs
cudaError_t launch_setup_host(MatPtr* tab, const float* const* hX, float* const* hQ, int B, uint32_t* maxbits,
                              int* status, cudaStream_t st);
cudaError_t launch_absmax(PtrArg p, int K, int r, long long ldx, int B, uint32_t* maxbits, cudaStream_t st);

// TMA tensor maps per matrix (128 bytes each, maps + (b * TMAPS_PER_MATRIX + m) * 128), 2-D fp32:
//   m = TMAP_X, TMAP_Q    tiles of TMAP_BOX_COLS x TMAP_BOX_ROWS (32 columns x 128 rows: one solve block)
//   m = TMAP_GX, TMAP_GQ  tiles of GRAM_BOX_COLS x GRAM_BOX_ROWS (128 columns x 32 rows: one Gram chunk)
// `any` is a 16-byte aligned device address for the host-side templates.
constexpr int TMAPS_PER_MATRIX = 4;
enum { TMAP_X = 0, TMAP_Q = 1, TMAP_GX = 2, TMAP_GQ = 3 };
constexpr int TMAP_BOX_COLS = 32;
constexpr int TMAP_BOX_ROWS = 128;
constexpr int GRAM_BOX_COLS = 128;
constexpr int GRAM_BOX_ROWS = 32;
// streaming multiprocessors of the current device (looked up once per device)
cudaError_t sm_count(int* nsm);
cudaError_t encode_rows(CUtensorMap* m, const void* base, int rows, int cols, long long ld, int box_cols, int box_rows);
cudaError_t launch_tmaps(PtrArg p, int K, int r, long long ldx, long long ldq, int B, const void* any, char* maps,
                         cudaStream_t st);

// tensor-core Gram: 128 x 128 tiles, splits of GRAM_TC_SPLIT rows (a multiple of 128); partials
// P[b][split][tile][128][128]; a bounded wait that runs out ORs 0x10 into *status
constexpr int GRAM_TC_SPLIT = 512;
GramPlan gram_tc_plan(int K, int n);
// mode GRAM_ACCURATE: exact three-way split and six products, the large-term accumulator drained into fp64 every 32
// rows (the reference's compensated Grams, for the component entry point); GRAM_DRAINED: two-way split, three
// products, drained every 128 rows (the last polish step: without the drains its truncating accumulation costs
// orthogonality); GRAM_PLAIN: two-way split, the whole split accumulated in TMEM
enum { GRAM_PLAIN = 0, GRAM_ACCURATE = 1, GRAM_DRAINED = 2 };
cudaError_t launch_gram_tc(PtrArg p, Src src, int K, int n, long long ld, int B, const GramPlan& gp, ScaleArg sc,
                           int accurate, float* P, int* status, cudaStream_t st);
// the two-way-split Gram for n <= 256, warp-specialised and fed by TMA (maps from launch_tmaps): one CTA per 128-row
// panel of G and split, N = n - 128 i columns wide; same partial layout; a bounded wait that runs out ORs 0x10
cudaError_t launch_gram_ws(PtrArg p, Src src, int K, int n, int B, const GramPlan& gp, const char* maps, ScaleArg sc,
                           float* P, int* status, cudaStream_t st);

// G[b] (n x n, both triangles) = fp64 sum over splits; with make_D, D = 0.5 (I - G) instead.  Without make_D (and sq
// not null) also sq[b * n + i], i < gram_sq_parts(gp) (<= n): fp64 partial sums of the squares of G's entries
int gram_sq_parts(const GramPlan& gp);
cudaError_t launch_gram_reduce(const float* P, int n, int B, const GramPlan& gp, int make_D, float* G, double* sq,
                               cudaStream_t st);

// Clamped Cholesky of A[b] (n x n, lower tiles read, overwritten).  Pipeline mode (sq != null): nrm = sqrt of the sum
// of sq[b * n + 0 .. nsq) in order, A_ii += 1e-7 nrm, tau = 1e-8 nrm + 1e-30, scalars to scal[b].  Component mode:
// tau = *tau_ptr, no shift.
cudaError_t launch_chol(float* A, float* L, float* Li, int n, int B, const double* sq, int nsq, const float* tau_ptr,
                        PassScal* scal, int zero_upper, cudaStream_t st);

// The solve's coefficient image W (W_jj = Li_j, W_jk = -Li_j L_jk, split tf32 tiles of 4 KB per part), grouped by
// block column k: [W_kk hi | W_kk lo | W_{k+1..nb-1, k} hi | W_{k+1..nb-1, k} lo]; wcol_off(nb, k) is the group's
// byte offset, wcol_off(nb, nb) = trsm_w_bytes(n) the size per matrix.
__host__ __device__ inline size_t wcol_off(int nb, int k) { return (size_t)(k * nb - k * (k - 1) / 2) * 2 * 4096; }
size_t trsm_w_bytes(int n);
cudaError_t launch_trsm_w(const float* L, const float* Li, int n, int B, char* W, cudaStream_t st);
// the same solve on the tensor cores from the image W, for the panel of blocks j0 .. j0 + nbp - 1 (nbp <= 8) of an
// n <= 512 matrix; input rows by the TMA maps (launch_tmaps), output to Q; `init` (K x 256 floats per matrix, or
// null) starts the panel's large accumulators; a bounded wait that runs out ORs 0x40 into *status
cudaError_t launch_trsm_tc(PtrArg p, Src src, int K, int n, long long ldq, int B, int j0, int nbp, const float* init,
                           const char* maps, const float* Z, long long ldz, ScaleArg sc, float eps, const char* W,
                           int* status, cudaStream_t st);
// scratch[b][row][0 .. 32 nbp) = sum_{k < j0} Y_k W_{j0.., k}^T (Y = the first 32 j0 columns of Q): the second
// panel's start for launch_trsm_tc; a bounded wait that runs out ORs 0x20 into *status
cudaError_t launch_trsm_panel_product(PtrArg p, int K, int n, long long ldq, int B, int j0, int nbp, const char* maps,
                                      const char* W, float* scratch, int* status, cudaStream_t st);

// Q <- Q + Q D per matrix, n <= 512, warp-specialised and fed by TMA (maps from launch_tmaps): D is first split into
// its operand image `img` (ns_dimg_bytes(n) per matrix); for n > 256 `scratch` holds K x 256 floats per matrix; a
// bounded wait that runs out ORs 0x20 into *status
__host__ __device__ inline size_t ns_dimg_bytes(int n) { return (size_t)8 * n * n; }
cudaError_t launch_ns_ws(PtrArg p, int K, int n, long long ldq, int B, const float* D, const char* maps, char* img,
                         float* scratch, int* status, cudaStream_t st);

// ---- block Gram-Schmidt (r > 512, 256-column blocks) ----
constexpr int BLOCK_W = 256;
// the band plan for T = P^T W with P = the first j columns and W the next 256 of a K-row matrix (splits of 2048 rows)
GramPlan gram_band_plan(int K, int j);
// -T as the update's operand image (B operand rows = W's 256 columns, contraction over P's j columns), from the band
// partials summed in split order (float-float): j x 256 x 8 bytes per matrix
__host__ __device__ inline size_t band_img_bytes(int j) { return (size_t)8 * j * BLOCK_W; }
cudaError_t launch_band_image(const float* P, const GramPlan& gp, int j, char* img, cudaStream_t st);
// Q[:, j .. j + 256) += Q[:, 0 .. j) (-T), in place, from that image (maps from launch_tmaps over Q); a bounded wait
// that runs out ORs 0x20 into *status
cudaError_t launch_project(PtrArg p, int K, int n, long long ldq, int j, const char* maps, const char* img,
                           int* status, cudaStream_t st);
// Q[:, 0 .. w) = s X[:, 0 .. w) with s = pow2_scale(max |X|) from *maxbits
cudaError_t launch_scale_copy(const float* X, long long ldx, float* Q, long long ldq, int K, int w,
                              const uint32_t* maxbits, cudaStream_t st);



}  // namespace spq
