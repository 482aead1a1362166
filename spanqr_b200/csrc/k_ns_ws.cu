// Newton-Schulz update Q <- Q + Q D (candidates/kcholqr.py:22, torch.addmm(Y, Y, D)) on the tcgen05 tensor cores,
// 3xTF32 (products hi.hi, hi.lo, lo.hi of the tf32 split of both operands).
//
// k_d_image splits D (symmetric, from k_gram_reduce) once per matrix into tf32 hi/lo operand tiles laid out as the
// update's shared-memory B operand: for each chunk of 32 contraction indices and each column half, the half's rows c
// (row c of D is column c) x 32 k, K-major with the 128-byte swizzle, hi part then lo part, so that the update streams
// each chunk of each half with one bulk copy.
// Warp roles of both kernels: 0-3 epilogue (TMEM lanes = rows: y + acc), 4-7 convert (raw 32-column tile of Q by TMA
// -> tf32 hi | lo, K-major), 8 products (one thread, fixed order), 9 copies (one thread).
// k_ns_pt (n <= 256, and the block projection): persistent, one CTA per SM over the 128-row tiles of the batch, two
// TMEM accumulators of 256 columns so that one tile's epilogue overlaps the next tile's products; the three products
// share an accumulator.
// k_ns_ws (n in (256, 512], and the solve's panel product): one CTA per 128-row tile, all n output columns in two
// column halves of N = n / 2 (TMEM holds the large (hi.hi) and small (hi.lo + lo.hi) accumulators of one half).  The
// last half is written in place; the first still feeds the second half's products, so its new values wait in
// `scratch` and are copied in after the last half.
// Product mode (k_ns_ws MODE 1, for the triangular solve of n > 256): the same pipeline computes only the accumulator
// sum_{k < j0} Y_k [W_{j0, k}; ...; W_{j0+nbp-1, k}]^T from the solve's W image (A = the first 32 j0 columns of Q,
// B = the stacked W tiles of block column k) and writes it to `scratch` (K x 256 per matrix).
// Projection (k_ns_pt<2>, block Gram-Schmidt for r > 512, candidates/kbig.py:66-95 W - P (P^T W)): A = the first j0
// columns of Q (the finished blocks P), B = -T (T = P^T W, k_band_image), N = 256; the result is added to the block
// W = Q[:, j0 .. j0 + 256) in place.
// Accuracy: |Q D| is about 1e-2 |Q| or less, so 3xTF32 and the truncating fp32 accumulation leave errors below one ulp
// of Q.
#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int NT = 320;
constexpr int ROWS = 128;
constexpr int CH = 32;                          // contraction indices per chunk
constexpr int YT = ROWS * CH * 4;               // 128 x 32 fp32 / tf32: 16 KB
constexpr int DPART = 256 * CH * 4;             // up to 256 rows of D x 32 k: 32 KB
constexpr int OFF_RAW = 0;                      // two raw A tiles
constexpr int OFF_AOP = OFF_RAW + 2 * YT;       // two A operand stages [hi | lo]
constexpr int OFF_DB = OFF_AOP + 2 * 2 * YT;    // two D operand stages [hi | lo]
constexpr int OFF_BAR = OFF_DB + 2 * 2 * DPART;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TCOLS = 512;                 // large at 0, small at 256
constexpr int ERR_TIMEOUT = 0x20;
// mbarriers (x2 per stage): raw A landed, raw A read (128 arrivals), A operands written (128 arrivals), D chunk
// landed, chunk products done; then a half's products done, its accumulators read (128 arrivals), error drain.
// Every waiter steps through a barrier's phases in order from phase 0, and no barrier can run two phases ahead of a
// waiter.
enum { B_RAW = 0, B_RAWFREE = 2, B_OP = 4, B_D = 6, B_FREE = 8, B_DONE = 10, B_TFREE = 11, B_FIN = 12, NBAR = 13 };
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(TMAP_BOX_COLS == CH && TMAP_BOX_ROWS == ROWS, "one TMA box is one 128-row tile of a chunk");
__device__ __forceinline__ uint32_t ring_parity(int c) { return (uint32_t)((c >> 1) & 1); }
}  // namespace

// one thread: row c of D, k-quad q of chunk kc
__global__ void k_d_image(const float* __restrict__ D_all, int n, char* __restrict__ img_all) {
    const int b = blockIdx.y;
    const int e = blockIdx.x * blockDim.x + threadIdx.x;   // (kc, c, q)
    const int nq = n / 4;
    if (e >= n * nq) return;
    const int c = e / nq, kq = e % nq, kc = kq / 8, q = kq % 8;
    const int N = n > 256 ? n / 2 : n, h = c / N, rr = c % N;   // column half and row within it
    const float4 v = *reinterpret_cast<const float4*>(D_all + (size_t)b * n * n + (size_t)c * n + 4 * kq);
    char* part = img_all + (size_t)b * ns_dimg_bytes(n) + (size_t)kc * 2 * n * 128 + (size_t)h * 2 * N * 128;
    tc::store2_at(part, part + (size_t)N * 128, tc::swz_off(rr, q), v);
}

template <int NH, int MODE>   // NH: column halves (1 for n <= 256, 2 above); MODE: 0 update, 1 solve panel product
__global__ void __launch_bounds__(NT, 1) k_ns_ws(PtrArg p, int K, int n, long long ldq, const char* __restrict__ maps,
                                                 const char* __restrict__ img_all, float* __restrict__ scratch,
                                                 int* __restrict__ status, int ncontr, int Nout, int j0) {
    extern __shared__ unsigned char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const RAW = sm + OFF_RAW;
    char* const AOP = sm + OFF_AOP;
    char* const DB = sm + OFF_DB;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 128);
    volatile int* err = reinterpret_cast<volatile int*>(sm + OFF_BAR + 132);

    const int b = blockIdx.y;
    const int row0 = blockIdx.x * ROWS;
    const int nchunks = ncontr / CH;              // chunks of the contraction
    constexpr int nh = NH;
    const int N = Nout;                           // width of a column half (MODE 1: of the panel product)
    const int total = nh * nchunks;               // chunks over all halves: g = h * nchunks + c
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i)
            tc::mbar_init(&bars[i], ((i >= B_RAWFREE && i < B_D) || i == B_TFREE) ? 128 : 1);
        tc::mbar_fence_init();
        *err = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        // ---------------- epilogue: row me, y + acc per half ----------------
        const int me = warp * 32 + lane, row = row0 + me;
        float* qr = (p.tab ? p.tab[b] : p.one).Q + (long long)row * ldq;
        float* sr = scratch ? scratch + ((size_t)b * K + (size_t)(row < K ? row : 0)) * 256 : nullptr;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        // the addend y (this row of Q before the update; nothing writes it before the last half's epilogue) is loaded
        // one 32-column block ahead: the first before the products are done, each next one during the current one
        const bool addend = MODE == 0 && row < K;
        const bool w8 = tc::al32(qr);   // 32-byte accesses where the row allows them (scratch rows always do)
        float yv[32], yn[32];
        auto load_y = [&](float (&y)[32], int col) {
            if (addend) {
                tc::ld_row32(qr + col, y, w8);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) y[i] = 0.f;
            }
        };
        for (int h = 0; h < nh; ++h) {
            const int c0 = h * N;
            load_y(yv, c0);
            const bool done = !*err && tc::mbar_wait_sleep(&bars[B_DONE], (uint32_t)(h & 1), 500);
            if (!__all_sync(0xffffffffu, done && !*err)) {   // per warp: tcgen05.ld needs the whole warp
                *err = 1;
                break;
            }
            tc::fence_after_sync();
            const bool to_scratch = MODE == 1 || (nh > 1 && h + 1 < nh);   // an earlier half waits in scratch
            float* dst = to_scratch ? sr : qr + c0;
            for (int cb = 0; cb < N / 32; ++cb) {
                if (cb + 1 < N / 32) load_y(yn, c0 + 32 * (cb + 1));
                float big[32], small[32];
                tc::tmem_ld32(tl + 32 * cb, big);
                tc::tmem_ld32(tl + 256 + 32 * cb, small);
                tc::tmem_wait_ld();
                if (row < K) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) big[i] = __fadd_rn(big[i], small[i]);
                    if (MODE == 0) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) big[i] = __fadd_rn(yv[i], big[i]);
                    }
                    tc::st_row32(dst + 32 * cb, big, to_scratch || w8);
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) yv[i] = yn[i];
            }
            if (nh > 1 && h + 1 < nh) {   // the next half's products may overwrite the accumulators
                tc::fence_before_sync();
                tc::mbar_arrive(&bars[B_TFREE]);
            }
        }
        if (MODE == 0 && nh > 1 && !*err && row < K) {   // every half's products have read this row: scratch goes in
            for (int c = 0; c < N; c += 32) {
                float v[32];
                tc::ld_row32(sr + c, v, true);
                tc::st_row32(qr + c, v, w8);
            }
        }
    } else if (warp < 8) {
        // ---------------- convert: raw Q tile -> tf32 hi | lo, rows 16 i + t / 8, k-quad t % 8 ----------------
        const int t = tid - 128, aq = t & 7, am = t >> 3;
        for (int c = 0; c < total; ++c) {   // c: chunk over all halves
            const int st = c & 1;
            if (*err || !tc::mbar_wait(&bars[B_RAW + st], ring_parity(c))) {
                *err = 1;
                break;
            }
            const char* raw = RAW + st * YT;
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = *reinterpret_cast<const float4*>(raw + 128 * (16 * i + am) + 16 * aq);
            // the next TMA load into this stage writes through the async proxy: order the generic reads above first
            tc::fence_async_smem();
            tc::mbar_arrive(&bars[B_RAWFREE + st]);
            if (c >= 2 && !tc::mbar_wait(&bars[B_FREE + st], ring_parity(c - 2))) {   // products of chunk c - 2 done
                *err = 1;
                break;
            }
            char* op = AOP + st * 2 * YT;
#pragma unroll
            for (int i = 0; i < 8; ++i) tc::store2_at(op, op + YT, tc::swz_off(16 * i + am, aq), v[i]);
            tc::fence_async_smem();
            tc::mbar_arrive(&bars[B_OP + st]);
        }
    } else if (warp == 8) {
        // ---------------- products ----------------
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_tf32(ROWS, N);
            bool ok = true;
            for (int g = 0; g < total; ++g) {
                const int st = g & 1, h = (nh > 1 && g >= nchunks) ? 1 : 0, c = g - h * nchunks;
                if (nh > 1 && c == 0 && h > 0) {   // the previous half's accumulators have been read
                    ok = !*err && tc::mbar_wait(&bars[B_TFREE], (uint32_t)((h - 1) & 1));
                    if (!ok) break;
                }
                ok = !*err && tc::mbar_wait(&bars[B_OP + st], ring_parity(g)) &&   // spin: the critical path
                     
                     tc::mbar_wait(&bars[B_D + st], ring_parity(g));
                if (!ok) break;
                tc::fence_after_sync();
                const uint32_t a = tc::smem_u32(AOP + st * 2 * YT), d = tc::smem_u32(DB + st * 2 * DPART);
#pragma unroll 1
                for (int k = 0; k < CH / 8; ++k) {
                    const uint64_t ahi = tc::sdesc_k128(a + 32 * k), alo = tc::sdesc_k128(a + YT + 32 * k);
                    const uint64_t dhi = tc::sdesc_k128(d + 32 * k), dlo = tc::sdesc_k128(d + N * 128 + 32 * k);
                    const uint32_t acc = (c > 0 || k > 0) ? 1u : 0u;
                    tc::mma_tf32(tmem, ahi, dhi, idesc, acc);
                    tc::mma_tf32(tmem + 256, ahi, dlo, idesc, acc);
                    tc::mma_tf32(tmem + 256, alo, dhi, idesc, 1u);
                }
                tc::mma_commit(&bars[B_FREE + st]);
                if (c == nchunks - 1) tc::mma_commit(&bars[B_DONE]);   // this half's products are done
            }
            if (!ok) {
                *err = 1;
                tc::mma_commit(&bars[B_FIN]);   // let issued products finish before TMEM is released
                tc::mbar_wait(&bars[B_FIN], 0u);
            }
        }
    } else {
        // ---------------- copies ----------------
        if (lane == 0) {
            const void* map = maps + ((size_t)b * TMAPS_PER_MATRIX + TMAP_Q) * 128;
            const char* img = img_all + (size_t)b * (MODE == 0 ? ns_dimg_bytes(n) : wcol_off(n / CH, n / CH));
            const uint32_t pbytes = (uint32_t)(N * 128);   // one half's rows of one part (hi or lo) of a D chunk
            tc::tmap_acquire(map);
            int n_raw[2] = {0, 0}, n_d[2] = {0, 0};
            bool ok = true;
            for (int g = 0; g < total; ++g) {
                const int st = g & 1, h = (nh > 1 && g >= nchunks) ? 1 : 0, c = g - h * nchunks;
                if (g >= 2) {
                    // raw tile g - 2 read by the convert warps; D chunk g - 2 read by its products
                    ok = !*err && tc::mbar_wait_sleep(&bars[B_RAWFREE + st], ring_parity(g - 2), 100) &&
                         tc::mbar_wait_sleep(&bars[B_FREE + st], ring_parity(g - 2), 100);
                    if (!ok) break;
                }
                tc::mbar_expect_tx(&bars[B_RAW + st], (uint32_t)YT);
                tc::tma_load_2d(RAW + st * YT, map, c * CH, row0, &bars[B_RAW + st]);
                ++n_raw[st];
                tc::mbar_expect_tx(&bars[B_D + st], 2 * pbytes);
                if (MODE == 0) {
                    const char* chunk = img + (size_t)c * 2 * n * 128 + (size_t)h * 2 * pbytes;   // hi rows, lo rows
                    tc::bulk_g2s(DB + st * 2 * DPART, chunk, 2 * pbytes, &bars[B_D + st]);
                } else {
                    // block column c of the W image: tiles j0 .. of its trailing list (hi), and the same in the lo list
                    const int NB = n / CH;
                    const char* hi = img + wcol_off(NB, c) + 2 * 4096 + (size_t)(j0 - c - 1) * 4096;
                    tc::bulk_g2s(DB + st * 2 * DPART, hi, pbytes, &bars[B_D + st]);
                    tc::bulk_g2s(DB + st * 2 * DPART + pbytes, hi + (size_t)(NB - 1 - c) * 4096, pbytes, &bars[B_D + st]);
                }
                ++n_d[st];
            }
            if (!ok) {
                *err = 1;
                for (int i = 0; i < 2; ++i) {   // let issued copies land before the shared memory is released
                    if (n_raw[i]) tc::mbar_wait(&bars[B_RAW + i], (uint32_t)((n_raw[i] - 1) & 1));
                    if (n_d[i]) tc::mbar_wait(&bars[B_D + i], (uint32_t)((n_d[i] - 1) & 1));
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0 && *err) atomicOr(status, ERR_TIMEOUT);
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

// Persistent form for at most 256 output columns (the update of n <= 256, the block projection): one CTA per SM loops
// over 128-row tiles (tile t = matrix t / nrb, row block t % nrb; CTA x takes t = x, x + grid, ...), the chunk rings
// run on from tile to tile, and TMEM holds two accumulators of 256 columns, so the epilogue of one tile overlaps the
// products of the next.  The three products of a k-step go into one accumulator: the result is y + Q D with
// |Q D| <= 1e-2 |Q| (the update) or the first projections of a block (repeated, BCGS2), so the truncating fp32 sum of
// the small products adds errors far below one ulp of the result.
// Two copy threads: raw Q tiles (HBM) are issued as soon as the convert warps have read the stage's previous tile, and
// the hi and lo parts of each B chunk (L2) as soon as the products that read the stage's previous parts are done:
// per chunk the products that read the lo part (hi.lo) go first and release it, then hi.hi and lo.hi.
namespace {
constexpr int NT_PT = 352;   // warps 0-3 epilogue, 4-7 convert, 8 products, 9 raw copies, 10 B copies
enum {
    P_RAW = 0, P_RAWFREE = 2, P_OP = 4, P_DHI = 6, P_DLO = 8, P_FREELO = 10, P_FREE = 12, P_DONE = 14, P_TFREE = 16,
    P_FIN = 18, P_NBAR = 19
};
static_assert(P_NBAR * 8 <= 128 + 64, "barriers below the TMEM slot");
}  // namespace

template <int MODE>   // 0: update, 2: projection
__global__ void __launch_bounds__(NT_PT, 1) k_ns_pt(PtrArg p, int K, long long ldq, const char* __restrict__ maps,
                                                    const char* __restrict__ img_all, int* __restrict__ status,
                                                    int ncontr, int N, int j0, int ntiles) {
    extern __shared__ unsigned char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const RAW = sm + OFF_RAW;
    char* const AOP = sm + OFF_AOP;
    char* const DB = sm + OFF_DB;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 192);
    volatile int* err = reinterpret_cast<volatile int*>(sm + OFF_BAR + 196);

    const int nrb = (K + ROWS - 1) / ROWS;
    const int nchunks = ncontr / CH;
    const int nloc = (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;   // this CTA's tiles
    const int total = nloc * nchunks;
    const int oc0 = MODE == 2 ? j0 : 0;   // the output's first column
    const size_t img_stride = MODE == 0 ? ns_dimg_bytes(N) : band_img_bytes(ncontr);
    const uint32_t pbytes = (uint32_t)(N * 128);   // one part (hi or lo) of a chunk of the B image
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    auto tile_of = [&](int i, int& b, int& row0) {
        const int t = (int)blockIdx.x + i * (int)gridDim.x;
        b = t / nrb;
        row0 = (t - b * nrb) * ROWS;
    };

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (tid == 0) {
        for (int i = 0; i < P_NBAR; ++i)
            tc::mbar_init(&bars[i], ((i >= P_RAWFREE && i < P_DHI) || (i >= P_TFREE && i < P_FIN)) ? 128 : 1);
        tc::mbar_fence_init();
        *err = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        // ---------------- epilogue: row me of each tile, y + acc ----------------
        const int me = warp * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        for (int i = 0; i < nloc; ++i) {
            const int buf = i & 1;
            int b, row0;
            tile_of(i, b, row0);
            const int row = row0 + me;
            const bool in = row < K;
            float* qr = (p.tab ? p.tab[b] : p.one).Q + (long long)(in ? row : 0) * ldq + oc0;
            const bool w8 = (reinterpret_cast<uintptr_t>(qr) & 31) == 0;   // 32-byte accesses where aligned
            // the addend y (this row before the update; nothing writes it before this epilogue) is loaded one
            // 32-column block ahead: the first before the products are done, each next one during the current one
            float yv[32], yn[32];
            auto load_y = [&](float (&y)[32], int col) {
                if (!in) {
#pragma unroll
                    for (int k = 0; k < 32; ++k) y[k] = 0.f;
                } else if (w8) {
#pragma unroll
                    for (int k = 0; k < 32; k += 8) tc::ld8(qr + col + k, y + k);
                } else {
#pragma unroll
                    for (int k = 0; k < 32; k += 4) {
                        const float4 t = *reinterpret_cast<const float4*>(qr + col + k);
                        y[k] = t.x, y[k + 1] = t.y, y[k + 2] = t.z, y[k + 3] = t.w;
                    }
                }
            };
            load_y(yv, 0);
            const bool done = !*err && tc::mbar_wait_sleep(&bars[P_DONE + buf], (uint32_t)((i >> 1) & 1), 200);
            if (!__all_sync(0xffffffffu, done && !*err)) {   // per warp: tcgen05.ld needs the whole warp
                *err = 1;
                break;
            }
            tc::fence_after_sync();
            for (int cb = 0; cb < N / 32; ++cb) {
                if (cb + 1 < N / 32) load_y(yn, 32 * (cb + 1));
                float acc[32];
                tc::tmem_ld32(tl + (uint32_t)(buf * 256 + 32 * cb), acc);
                tc::tmem_wait_ld();
                if (in) {
#pragma unroll
                    for (int k = 0; k < 32; ++k) acc[k] = __fadd_rn(yv[k], acc[k]);
                    if (w8) {
#pragma unroll
                        for (int k = 0; k < 32; k += 8) tc::st8(qr + 32 * cb + k, acc + k);
                    } else {
#pragma unroll
                        for (int k = 0; k < 32; k += 4)
                            *reinterpret_cast<float4*>(qr + 32 * cb + k) = make_float4(acc[k], acc[k + 1], acc[k + 2], acc[k + 3]);
                    }
                }
#pragma unroll
                for (int k = 0; k < 32; ++k) yv[k] = yn[k];
            }
            tc::fence_before_sync();
            tc::mbar_arrive(&bars[P_TFREE + buf]);   // the next products into this buffer may start
        }
    } else if (warp < 8) {
        // ---------------- convert: raw Q tile -> tf32 hi | lo, rows 16 i + t / 8, k-quad t % 8 ----------------
        const int t = tid - 128, aq = t & 7, am = t >> 3;
        for (int g = 0; g < total; ++g) {
            const int st = g & 1;
            if (*err || !tc::mbar_wait(&bars[P_RAW + st], ring_parity(g))) {
                *err = 1;
                break;
            }
            const char* raw = RAW + st * YT;
            float4 v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = *reinterpret_cast<const float4*>(raw + 128 * (16 * k + am) + 16 * aq);
            // the next TMA load into this stage writes through the async proxy: order the generic reads above first
            tc::fence_async_smem();
            tc::mbar_arrive(&bars[P_RAWFREE + st]);
            if (g >= 2 && !tc::mbar_wait(&bars[P_FREE + st], ring_parity(g - 2))) {   // products of chunk g - 2 done
                *err = 1;
                break;
            }
            char* op = AOP + st * 2 * YT;
#pragma unroll
            for (int k = 0; k < 8; ++k) tc::store2_at(op, op + YT, tc::swz_off(16 * k + am, aq), v[k]);
            tc::fence_async_smem();
            tc::mbar_arrive(&bars[P_OP + st]);
        }
    } else if (warp == 8) {
        // ---------------- products ----------------
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_tf32(ROWS, N);
            bool ok = true;
            int g = 0;
            for (int i = 0; i < nloc && ok; ++i) {
                const int buf = i & 1;
                const uint32_t acc = tmem + (uint32_t)(buf * 256);
                if (i >= 2) {   // the epilogue has read this buffer's previous tile
                    ok = !*err && tc::mbar_wait(&bars[P_TFREE + buf], (uint32_t)(((i - 2) >> 1) & 1));
                    if (!ok) break;
                    tc::fence_after_sync();
                }
                for (int c = 0; c < nchunks; ++c, ++g) {
                    const int st = g & 1;
                    const uint32_t a = tc::smem_u32(AOP + st * 2 * YT), d = tc::smem_u32(DB + st * 2 * DPART);
                    ok = !*err && tc::mbar_wait(&bars[P_OP + st], ring_parity(g)) &&
                         tc::mbar_wait(&bars[P_DLO + st], ring_parity(g));
                    if (!ok) break;
                    tc::fence_after_sync();
#pragma unroll 1
                    for (int k = 0; k < CH / 8; ++k)   // hi.lo: releases the lo part
                        tc::mma_tf32(acc, tc::sdesc_k128(a + 32 * k), tc::sdesc_k128(d + pbytes + 32 * k), idesc,
                                     (c > 0 || k > 0) ? 1u : 0u);
                    tc::mma_commit(&bars[P_FREELO + st]);
                    ok = !*err && tc::mbar_wait(&bars[P_DHI + st], ring_parity(g));
                    if (!ok) break;
                    tc::fence_after_sync();
#pragma unroll 1
                    for (int k = 0; k < CH / 8; ++k) {   // hi.hi, lo.hi
                        const uint64_t dhi = tc::sdesc_k128(d + 32 * k);
                        tc::mma_tf32(acc, tc::sdesc_k128(a + 32 * k), dhi, idesc, 1u);
                        tc::mma_tf32(acc, tc::sdesc_k128(a + YT + 32 * k), dhi, idesc, 1u);
                    }
                    tc::mma_commit(&bars[P_FREE + st]);
                }
                if (ok) tc::mma_commit(&bars[P_DONE + buf]);   // this tile's products are done
            }
            if (!ok) {
                *err = 1;
                tc::mma_commit(&bars[P_FIN]);   // let issued products finish before TMEM is released
                tc::mbar_wait(&bars[P_FIN], 0u);
            }
        }
    } else if (warp == 9) {
        // ---------------- raw Q tiles ----------------
        if (lane == 0) {
            int n_raw[2] = {0, 0};
            int cur = -1;
            bool ok = true;
            for (int g = 0; g < total; ++g) {
                const int st = g & 1, i = g / nchunks, c = g - i * nchunks;
                int b, row0;
                tile_of(i, b, row0);
                if (g >= 2) {   // raw tile g - 2 read by the convert warps
                    ok = !*err && tc::mbar_wait_sleep(&bars[P_RAWFREE + st], ring_parity(g - 2), 50);
                    if (!ok) break;
                }
                const void* map = maps + ((size_t)b * TMAPS_PER_MATRIX + TMAP_Q) * 128;
                if (b != cur) {
                    tc::tmap_acquire(map);
                    cur = b;
                }
                tc::mbar_expect_tx(&bars[P_RAW + st], (uint32_t)YT);
                tc::tma_load_2d(RAW + st * YT, map, c * CH, row0, &bars[P_RAW + st]);
                ++n_raw[st];
            }
            if (!ok) {
                *err = 1;
                for (int k = 0; k < 2; ++k)   // let issued copies land before the shared memory is released
                    if (n_raw[k]) tc::mbar_wait(&bars[P_RAW + k], (uint32_t)((n_raw[k] - 1) & 1));
            }
        }
    } else {
        // ---------------- B chunks: lo part, then hi part ----------------
        if (lane == 0) {
            int n_lo[2] = {0, 0}, n_hi[2] = {0, 0};
            bool ok = true;
            for (int g = 0; g < total; ++g) {
                const int st = g & 1, i = g / nchunks, c = g - i * nchunks;
                int b, row0;
                tile_of(i, b, row0);
                const char* chunk = img_all + (size_t)b * img_stride + (size_t)c * 2 * pbytes;   // hi rows, lo rows
                char* dst = DB + st * 2 * DPART;
                if (g >= 2) {   // the products of chunk g - 2 that read the lo part
                    ok = !*err && tc::mbar_wait_sleep(&bars[P_FREELO + st], ring_parity(g - 2), 50);
                    if (!ok) break;
                }
                tc::mbar_expect_tx(&bars[P_DLO + st], pbytes);
                tc::bulk_g2s(dst + pbytes, chunk + pbytes, pbytes, &bars[P_DLO + st]);
                ++n_lo[st];
                if (g >= 2) {   // all products of chunk g - 2
                    ok = !*err && tc::mbar_wait_sleep(&bars[P_FREE + st], ring_parity(g - 2), 50);
                    if (!ok) break;
                }
                tc::mbar_expect_tx(&bars[P_DHI + st], pbytes);
                tc::bulk_g2s(dst, chunk, pbytes, &bars[P_DHI + st]);
                ++n_hi[st];
            }
            if (!ok) {
                *err = 1;
                for (int k = 0; k < 2; ++k) {   // let issued copies land before the shared memory is released
                    if (n_lo[k]) tc::mbar_wait(&bars[P_DLO + k], (uint32_t)((n_lo[k] - 1) & 1));
                    if (n_hi[k]) tc::mbar_wait(&bars[P_DHI + k], (uint32_t)((n_hi[k] - 1) & 1));
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0 && *err) atomicOr(status, ERR_TIMEOUT);
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

template <int MODE>
static cudaError_t launch_pt(PtrArg p, int K, long long ldq, int B, const char* maps, const char* img, int* status,
                             int ncontr, int N, int j0, cudaStream_t st) {
    int nsm = 0;
    cudaError_t e = sm_count(&nsm);
    if (e != cudaSuccess) return e;
    const long long ntiles = (long long)cdiv(K, ROWS) * B;
    if (ntiles > (1LL << 30)) return cudaErrorInvalidValue;
    e = cudaFuncSetAttribute(k_ns_pt<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const int grid = (int)(ntiles < nsm ? ntiles : nsm);
    k_ns_pt<MODE><<<grid, NT_PT, SMEM_BYTES, st>>>(p, K, ldq, maps, img, status, ncontr, N, j0, (int)ntiles);
    return cudaGetLastError();
}

template <int NH, int MODE>
static cudaError_t launch_k(PtrArg p, int K, int n, long long ldq, int B, const char* maps, const char* img,
                            float* scratch, int* status, int ncontr, int N, int j0, cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(k_ns_ws<NH, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    k_ns_ws<NH, MODE><<<dim3(cdiv(K, ROWS), B), NT, SMEM_BYTES, st>>>(p, K, n, ldq, maps, img, scratch, status, ncontr,
                                                                     N, j0);
    return cudaGetLastError();
}

cudaError_t launch_ns_ws(PtrArg p, int K, int n, long long ldq, int B, const float* D, const char* maps, char* img,
                         float* scratch, int* status, cudaStream_t st) {
    if (n > 512 || n % CH || (n > 256 && !scratch)) return cudaErrorInvalidValue;
    k_d_image<<<dim3(cdiv(n * n / 4, 256), B), 256, 0, st>>>(D, n, img);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return n > 256 ? launch_k<2, 0>(p, K, n, ldq, B, maps, img, scratch, status, n, n / 2, 0, st)
                   : launch_pt<0>(p, K, ldq, B, maps, img, status, n, n, 0, st);
}

cudaError_t launch_trsm_panel_product(PtrArg p, int K, int n, long long ldq, int B, int j0, int nbp, const char* maps,
                                      const char* W, float* scratch, int* status, cudaStream_t st) {
    if (n > 512 || n % CH || j0 < 1 || nbp < 1 || nbp > 8 || (j0 + nbp) * CH > n || !scratch) return cudaErrorInvalidValue;
    return launch_k<1, 1>(p, K, n, ldq, B, maps, W, scratch, status, j0 * CH, nbp * CH, j0, st);
}

cudaError_t launch_project(PtrArg p, int K, int n, long long ldq, int j, const char* maps, const char* img,
                           int* status, cudaStream_t st) {
    if (j < BLOCK_W || j % BLOCK_W || j + BLOCK_W > n || ldq < n) return cudaErrorInvalidValue;
    return launch_pt<2>(p, K, ldq, 1, maps, img, status, j, BLOCK_W, j, st);
}

}  // namespace spq
