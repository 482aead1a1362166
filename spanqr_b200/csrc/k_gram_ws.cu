// Gram partials of Y (or s X) for n <= 256 on the tcgen05 tensor cores, two-way split TF32 (hi.hi + hi.lo + lo.hi):
// the Grams the reference computes as plain fp32 GEMMs (passes 2 and 3, the first polish step: kcholqr.py:106 and
// :20) and the first pass's compensated gram_f (tri.py:324-375), which the two-way split matches closely enough for
// every robustness and span test.
//
// Work item = one 128-row panel i of G over one split of GRAM_TC_SPLIT rows of Y: it computes
//     G[128 i .. 128 i + 127, 128 i .. n) over the split's rows
// as one M = 128, N = n - 128 i (<= 256) product per k-step.  A (the panel's 128 columns of Y) is the first 128
// columns of B (columns 128 i .. n of Y), so one staged chunk of 32 rows serves both operands, MN-major in the 32-byte
// base 128B-swizzled layout tcgen05 takes for 32-bit types.  The split accumulates in TMEM (hi.hi and the cross terms
// in separate accumulators) and is written to the partial tiles P[b][split][tile] of k_gram_tc (the same layout, so
// k_gram_reduce sums them unchanged); the tile diagonal is replaced by the sum of squares kept in float-float (exact
// squares, about 44 bits).
// Persistent: one CTA per SM walks the items (the two panels of a split side by side, every CTA alternating panels
// from round to round); the chunk rings run on from item to item, so the next item's copies and conversions proceed
// during an item's epilogue, and the products resume as soon as the epilogue has read the accumulators out of TMEM.
// Each item's arithmetic is the same whichever CTA computes it.
// Warp roles: 0-3 epilogue (float-float squares of the panel's columns from each raw chunk, then TMEM lanes = the
// panel's columns), 4-7 convert (raw chunk -> s y -> tf32 hi | lo), 8 products (one thread), 9 copies (one thread,
// TMA through the per-matrix maps).
#include "kernels.h"
#include "tc.cuh"

namespace spq {

namespace {
constexpr int NT = 320;
constexpr int TILE = 128;
constexpr int CH = 32;                       // rows per chunk (4 k-steps of 8)
constexpr int RAWB = GRAM_BOX_COLS * CH * 4; // one raw box: 128 columns x 32 rows fp32 = 16 KB
constexpr int RAW_STAGE = 2 * RAWB;          // up to two boxes (256 columns)
constexpr int OP_PART = 256 * CH * 4;        // one operand part (hi or lo) of up to 256 columns: 32 KB
constexpr int OP_STAGE = 2 * OP_PART;
constexpr int RSTAGES = 3;                   // raw chunks in flight (copies three chunks ahead of the conversion)
constexpr int OSTAGES = 2;                   // operand chunks
constexpr int OFF_RAW = 0;
constexpr int OFF_OP = OFF_RAW + RSTAGES * RAW_STAGE;
constexpr int OFF_BAR = OFF_OP + OSTAGES * OP_STAGE;
constexpr int OFF_DSQ = OFF_BAR + 256;       // an item's 128 column sums of squares (fp64)
constexpr int SMEM_BYTES = OFF_DSQ + TILE * 8 + 1024;
constexpr uint32_t TCOLS = 512;              // large at 0, small at 256
constexpr int ERR_TIMEOUT = 0x10;
// mbarriers (per stage where doubled): raw chunk landed, raw chunk read (128 arrivals), operands written (128
// arrivals), operands consumed, all products done, error drain.  Every waiter steps through a barrier's phases in
// order from phase 0, and no barrier can run two phases ahead of a waiter.
// a raw chunk is read by the convert warps and the epilogue warps (256 arrivals); per item: its products done, its
// accumulators read (128 arrivals)
enum { B_RAW = 0, B_RAWFREE = 3, B_OP = 6, B_OPFREE = 8, B_DONE = 10, B_TFREE = 11, B_FIN = 12, NBAR = 13 };
static_assert(NBAR * 8 <= 128, "barriers below the TMEM slot");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(GRAM_BOX_ROWS == CH && GRAM_BOX_COLS == TILE, "one TMA box is 128 columns of one chunk");

__device__ __forceinline__ uint32_t ring_parity(int c) { return (uint32_t)((c >> 1) & 1); }   // c-th use of a 2-ring
__device__ __forceinline__ uint32_t par3(int c) { return (uint32_t)((c / 3) & 1); }            // c-th use of a 3-ring

// byte offset of (k, mn .. mn+3) in an operand part whose MN extent is `w` (a multiple of 128): 32-byte-base layout,
// atoms of 4 k-rows x 32 MN (512 bytes) with the 32-byte granule g of k-row r at granule position g ^ r, MN-atoms
// 512 bytes apart, k-atoms 16 w bytes apart
__device__ __forceinline__ uint32_t mn_off(int k, int mn, int w) {
    const int kr = k & 3, g = (mn >> 3) & 3;
    return (uint32_t)((k >> 2) * (16 * w) + (mn >> 5) * 512 + kr * 128 + ((g ^ kr) << 5) + ((mn & 7) << 2));
}
}  // namespace

__global__ void __launch_bounds__(NT, 1) k_gram_ws(PtrArg p, Src src, int K, int n, GramPlan gp,
                                                   const char* __restrict__ maps, ScaleArg sc, float* __restrict__ P,
                                                   int* __restrict__ status, int items) {
    extern __shared__ unsigned char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    char* const RAW = sm + OFF_RAW;
    char* const OP = sm + OFF_OP;
    double* const DSQ = reinterpret_cast<double*>(sm + OFF_DSQ);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 128);
    volatile int* err = reinterpret_cast<volatile int*>(sm + OFF_BAR + 132);

    const int nloc = (items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;   // this CTA's items
    // item i of this CTA: panel pi, matrix b, split sp; its width, boxes, first row and chunks
    struct Item {
        int pi, b, sp, N, nbox, W, k0, nchunks;
    };
    auto item = [&](int i) {
        Item it;
        const int t = (int)blockIdx.x + i * (int)gridDim.x;
        // items 2u and 2u + 1 are the two panels of one split (so they run side by side and share its rows in L2),
        // their order flipped from one round of the grid to the next (so every CTA alternates panels)
        int u = t;
        it.pi = 0;
        if (gp.nt == 2) {
            u = t >> 1;
            it.pi = (t & 1) ^ (((t & ~1) / (int)gridDim.x) & 1);
        }
        it.b = u / gp.S;
        it.sp = u - it.b * gp.S;
        it.N = n - it.pi * TILE;
        it.nbox = it.N > TILE ? 2 : 1;
        it.W = it.nbox * TILE;
        it.k0 = it.sp * gp.KS;
        it.nchunks = (min(it.k0 + gp.KS, K) - it.k0 + CH - 1) / CH;
        return it;
    };
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (warp == 0) tc::tmem_alloc(tmem_slot, TCOLS);
    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i)   // raw read (256), operands written (128), accumulators read (128)
            tc::mbar_init(&bars[i], (i >= B_RAWFREE && i < B_OP) ? 256 : ((i >= B_OP && i < B_OPFREE) || i == B_TFREE) ? 128 : 1);
        tc::mbar_fence_init();
        *err = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        // ---------------- epilogue: squares of the panel's columns, then row a of tile row-panel pi (TMEM lane a) ------
        // squares: rows 8 warp .. + 7 of each chunk, columns 4 lane .. + 3 of the panel (the first box), float-float
        const int a = warp * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        int g = 0;   // chunk over all items
        for (int i = 0; i < nloc; ++i) {
            const Item it = item(i);
            float s = 1.0f;
            bool scaled = false;
            if (sc.maxbits) {
                s = pow2_scale(__uint_as_float(sc.maxbits[it.b]));
                scaled = true;
            } else if (sc.s) {
                s = sc.s[it.b];
                scaled = true;
            }
            float sqh[4] = {0.f, 0.f, 0.f, 0.f}, sql[4] = {0.f, 0.f, 0.f, 0.f};
            bool ok = true;
            for (int c = 0; c < it.nchunks; ++c, ++g) {
                const int rs = g % RSTAGES;
                if (*err || !tc::mbar_wait(&bars[B_RAW + rs], par3(g))) {
                    ok = false;
                    break;
                }
                const char* raw = RAW + rs * RAW_STAGE;
                float4 v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = *reinterpret_cast<const float4*>(raw + (8 * warp + k) * 512 + 16 * lane);
                tc::fence_async_smem();   // generic reads before the next TMA write into the stage
                tc::mbar_arrive(&bars[B_RAWFREE + rs]);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    float4 x = v[k];
                    if (scaled) {
                        x.x = __fmul_rn(x.x, s); x.y = __fmul_rn(x.y, s); x.z = __fmul_rn(x.z, s); x.w = __fmul_rn(x.w, s);
                    }
                    ff_add_sq(sqh[0], sql[0], x.x);
                    ff_add_sq(sqh[1], sql[1], x.y);
                    ff_add_sq(sqh[2], sql[2], x.z);
                    ff_add_sq(sqh[3], sql[3], x.w);
                }
            }
            // the item's column sums of squares: the warps' partial sums added in fp64 in warp order 0..3 (the four
            // warps leave together or not at all: they meet at named barriers below)
            if (!tc::bar_and(2, 128, ok)) {
                *err = 1;
                break;
            }
            for (int w = 0; w < 4; ++w) {
                tc::bar_sync(2, 128);
                if (warp == w) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        double* dq = &DSQ[4 * lane + j];
                        *dq = __dadd_rn(w == 0 ? 0.0 : *dq, ff_value(sqh[j], sql[j]));
                    }
                }
            }
            tc::bar_sync(2, 128);
            const double d = DSQ[a];
            const bool done = !*err && tc::mbar_wait_sleep(&bars[B_DONE], (uint32_t)(i & 1), 200);
            // one decision for the four warps (tcgen05.ld needs whole warps; the next item's barriers need all four)
            if (!tc::bar_and(2, 128, done && !*err)) {
                *err = 1;
                break;
            }
            tc::fence_after_sync();
            float* Pb = P + (size_t)(it.b * gp.S + it.sp) * gp.tiles * TILE * TILE;
            for (int cb = 0; cb < it.W / 32; ++cb) {
                float big[32], small[32];
                tc::tmem_ld32(tl + 32 * cb, big);
                tc::tmem_ld32(tl + 256 + 32 * cb, small);
                tc::tmem_wait_ld();
                const int tj = it.pi + (32 * cb) / TILE, c0 = (32 * cb) % TILE;
                const int t = it.pi * gp.nt - it.pi * (it.pi - 1) / 2 + (tj - it.pi);
                float* row = Pb + (size_t)t * TILE * TILE + (size_t)a * TILE + c0;
#pragma unroll
                for (int k = 0; k < 32; ++k) big[k] = __fadd_rn(big[k], small[k]);
                if (tj == it.pi && a >= c0 && a < c0 + 32) {
#pragma unroll
                    for (int k = 0; k < 32; ++k)
                        if (c0 + k == a) big[k] = __double2float_rn(d);
                }
                tc::st_row32(row, big, true);   // partial rows: 512 bytes apart, 256-byte aligned base
            }
            tc::fence_before_sync();
            tc::mbar_arrive(&bars[B_TFREE]);   // the next item's products may overwrite the accumulators
        }
    } else if (warp < 8) {
        // ---------------- convert: rows 8 (warp - 4) .. +7 of each chunk, columns 4 lane .. of each box ----------------
        const int cw = warp - 4;
        int g = 0;   // chunk over all items
        bool ok = true;
        for (int i = 0; i < nloc && ok; ++i) {
            const Item it = item(i);
            float s = 1.0f;
            bool scaled = false;
            if (sc.maxbits) {
                s = pow2_scale(__uint_as_float(sc.maxbits[it.b]));
                scaled = true;
            } else if (sc.s) {
                s = sc.s[it.b];
                scaled = true;
            }
            for (int c = 0; c < it.nchunks; ++c, ++g) {
                const int st = g & 1, rs = g % RSTAGES;
                if (*err || !tc::mbar_wait(&bars[B_RAW + rs], par3(g))) {
                    ok = false;
                    break;
                }
                const char* raw = RAW + rs * RAW_STAGE;
                float4 v[2][8];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (h < it.nbox) {
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            v[h][k] = *reinterpret_cast<const float4*>(raw + h * RAWB + (8 * cw + k) * 512 + 16 * lane);
                    }
                }
                // the raw stage is released after the one proxy fence below: the next TMA load into it writes through
                // the async proxy, so these generic reads must be ordered before it by that fence (without one, bytes
                // of a later chunk were seen in place of chunk c's)
                if (scaled) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (h < it.nbox) {
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                float4& x = v[h][k];
                                x.x = __fmul_rn(x.x, s); x.y = __fmul_rn(x.y, s); x.z = __fmul_rn(x.z, s); x.w = __fmul_rn(x.w, s);
                            }
                        }
                    }
                }
                if (g >= 2 && !tc::mbar_wait(&bars[B_OPFREE + st], ring_parity(g - 2))) {   // products of g - 2 done
                    ok = false;
                    break;
                }
                char* op = OP + st * OP_STAGE;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (h < it.nbox) {
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const uint32_t o = mn_off(8 * cw + k, h * TILE + 4 * lane, it.W);
                            tc::store2_at(op, op + OP_PART, o, v[h][k]);
                        }
                    }
                }
                tc::fence_async_smem();
                tc::mbar_arrive(&bars[B_RAWFREE + rs]);
                tc::mbar_arrive(&bars[B_OP + st]);
            }
        }
        if (!ok) *err = 1;
    } else if (warp == 8) {
        // ---------------- products ----------------
        if (lane == 0) {
            bool ok = true;
            int g = 0;
            for (int i = 0; i < nloc && ok; ++i) {
                const Item it = item(i);
                const uint32_t idesc = tc::idesc_tf32_mn(TILE, it.N);
                if (i >= 1) {   // the epilogue has read the previous item's accumulators
                    ok = !*err && tc::mbar_wait(&bars[B_TFREE], (uint32_t)((i - 1) & 1));
                    if (!ok) break;
                    tc::fence_after_sync();
                }
                for (int c = 0; c < it.nchunks; ++c, ++g) {
                    const int st = g & 1;
                    ok = !*err && tc::mbar_wait(&bars[B_OP + st], ring_parity(g));   // spin: the critical path
                    if (!ok) break;
                    tc::fence_after_sync();
                    const uint32_t hi = tc::smem_u32(OP + st * OP_STAGE), lo = hi + OP_PART;
#pragma unroll 1
                    for (int k = 0; k < CH / 8; ++k) {
                        const uint32_t ko = (uint32_t)(2 * 16 * it.W * k);   // two k-atoms per k-step of 8
                        const uint64_t ahi = tc::sdesc_mn128b32(hi + ko, 512, 16 * it.W);
                        const uint64_t alo = tc::sdesc_mn128b32(lo + ko, 512, 16 * it.W);
                        const uint32_t acc = (c > 0 || k > 0) ? 1u : 0u;
                        tc::mma_tf32(tmem, ahi, ahi, idesc, acc);          // A and B share the staged columns
                        tc::mma_tf32(tmem + 256, ahi, alo, idesc, acc);
                        tc::mma_tf32(tmem + 256, alo, ahi, idesc, 1u);
                    }
                    tc::mma_commit(&bars[B_OPFREE + st]);
                }
                if (ok) tc::mma_commit(&bars[B_DONE]);
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
            int issued[RSTAGES] = {0, 0, 0};
            int cur = -1;
            bool ok = true;
            int g = 0;
            for (int i = 0; i < nloc && ok; ++i) {
                const Item it = item(i);
                const void* map = maps + ((size_t)it.b * TMAPS_PER_MATRIX + (src == SRC_X ? TMAP_GX : TMAP_GQ)) * 128;
                if (it.b != cur) {
                    tc::tmap_acquire(map);
                    cur = it.b;
                }
                for (int c = 0; c < it.nchunks; ++c, ++g) {
                    const int rs = g % RSTAGES;
                    if (g >= RSTAGES) {
                        ok = !*err && tc::mbar_wait_sleep(&bars[B_RAWFREE + rs], par3(g - RSTAGES), 100);   // g - 3 read
                        if (!ok) break;
                    }
                    tc::mbar_expect_tx(&bars[B_RAW + rs], (uint32_t)(it.nbox * RAWB));
                    for (int h = 0; h < it.nbox; ++h)
                        tc::tma_load_2d(RAW + rs * RAW_STAGE + h * RAWB, map, it.pi * TILE + h * TILE, it.k0 + c * CH,
                                        &bars[B_RAW + rs]);
                    ++issued[rs];
                }
            }
            if (!ok) {
                *err = 1;
                for (int k = 0; k < RSTAGES; ++k)   // let issued copies land before the shared memory is released
                    if (issued[k]) tc::mbar_wait(&bars[B_RAW + k], (uint32_t)((issued[k] - 1) & 1));
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0 && *err) atomicOr(status, ERR_TIMEOUT);
    if (warp == 0) tc::tmem_dealloc(tmem, TCOLS);
}

cudaError_t launch_gram_ws(PtrArg p, Src src, int K, int n, int B, const GramPlan& gp, const char* maps, ScaleArg sc,
                           float* P, int* status, cudaStream_t st) {
    if (n > 2 * TILE || n % 32 || gp.KS % CH || gp.b0 != 0) return cudaErrorInvalidValue;
    int nsm = 0;
    cudaError_t e = sm_count(&nsm);
    if (e != cudaSuccess) return e;
    const long long items = (long long)gp.nt * gp.S * B;
    if (items > (1LL << 30)) return cudaErrorInvalidValue;
    e = cudaFuncSetAttribute(k_gram_ws, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const int grid = (int)(items < nsm ? items : nsm);
    k_gram_ws<<<grid, NT, SMEM_BYTES, st>>>(p, src, K, n, gp, maps, sc, P, status, (int)items);
    return cudaGetLastError();
}

}  // namespace spq
