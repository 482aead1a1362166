/*
 * spanqr_b200 -- C ABI of the B200-native orth(X) (libspanqr.so).
 *
 * orth(X): an orthonormal basis Q of the column span of a tall fp32 matrix X [K, r] (K >= r), by the robust
 * shifted Cholesky-QR recipe of oguzeldereli/spanqr (power-of-2 scale, seeded dust, three shifted and clamped
 * Cholesky-QR passes with blocked triangular solves, two Newton-Schulz polish steps).
 *
 * Conventions for every entry point:
 *   - all matrix pointers are DEVICE pointers on the current CUDA device, row-major fp32, 16-byte aligned, with
 *     leading dimensions (in elements) that are multiples of 4;
 *   - work is enqueued on `stream` (a cudaStream_t; NULL = legacy default stream) and never synchronises the host;
 *   - the caller owns every buffer, including the workspace `ws` (size from spanqr_workspace_bytes, 256-byte
 *     aligned); the library allocates no device memory on these paths;
 *   - calls in flight at the same time (on different streams or threads) need different workspaces;
 *   - the return value is SPANQR_OK or an error code (spanqr_strerror); nothing is enqueued on an error.
 *
 * Reference interfaces these replace (file:line in oguzeldereli/spanqr):
 *   spanqr_orth_f32          orth.py:13-20 -> candidates/kcholqr.py:92-112 kcholqr_f(X)
 *   spanqr_orth_strided_f32  no reference counterpart: a batch of same-shape layers (orth_batched)
 *   spanqr_orth_batched_f32  no reference counterpart: same, from device arrays of matrix pointers
 *   spanqr_orth_ptrs_f32     no reference counterpart: same, from host arrays of matrix pointers
 *   spanqr_orth_graph_*      no reference counterpart: spanqr_orth_f32 captured once per shape, replayed per call
 *   spanqr_orth_mixed_f32    no reference counterpart: a batch of layers of one width and different heights
 *   spanqr_borth_f32         orth.py:18-19 -> candidates/kbig.py:66-95 borth(X, b=256) (r > 512)
 *   spanqr_gram_f32          candidates/tri.py:362-375 gram_f(Y, s) and tri.py:285-297 gram_split(Y, bt=64)
 *   spanqr_gram_mode_f32     the same, and kcholqr.py:106 Y.T @ Y (each Gram of the orth sequence on its own)
 *   spanqr_chol_f32          candidates/kchol.py:35-44 chol32(G, tau) (kernel candidates/cuk/chol.cu:273-276)
 *   spanqr_trsm_f32          candidates/tri.py:406-412 trsm_f(X, L, Li, s, Z, eps)
 */
#ifndef SPANQR_H
#define SPANQR_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* spanqr_stream_t; /* the same type as cudaStream_t */

enum spanqr_status {
    SPANQR_OK = 0,
    SPANQR_ERR_SHAPE = 1,     /* r not a multiple of 32, r > 512, K < r, batch < 1 (no Householder fallback)   */
    SPANQR_ERR_ARG = 2,       /* null or misaligned pointer, leading dimension too small or not a multiple of 4 */
    SPANQR_ERR_WORKSPACE = 3, /* workspace too small or not 256-byte aligned                                    */
    SPANQR_ERR_CUDA = 4,      /* a CUDA runtime call or kernel launch failed                                    */
    SPANQR_ERR_DEVICE = 5,    /* the device status word reports a failure (spanqr_read_status)                  */
    SPANQR_ERR_TOO_LARGE = 6  /* the shape needs more scratch than spanqr_orth_noalloc_f32's fixed array holds     */
};

/* version as MAJOR * 10000 + MINOR * 100 + PATCH */
int spanqr_version(void);

/* human-readable text for a status code */
const char* spanqr_strerror(int code);

/* text of the last CUDA error seen by this library on the calling thread ("" if none) */
const char* spanqr_last_cuda_error(void);

/* Bytes of workspace a call with `batch` matrices of shape K x r needs (the same for orth, strided and batched). */
int spanqr_workspace_bytes(int K, int r, int batch, size_t* bytes);

/*
 * Q = orth(X).  X [K, r] (leading dimension ldx) is read only; Q [K, r] (ldq) is written.  Z [K, r] (leading
 * dimension r) is the dust: the reference draws it once per shape with torch.randn on the CUDA generator seeded
 * 20261018 and divides each column by its norm (kcholqr.py:83-89); the caller passes it in.
 */
int spanqr_orth_f32(const float* X, long long ldx, float* Q, long long ldq, int K, int r, const float* Z,
                    void* ws, size_t ws_bytes, spanqr_stream_t stream);

/* orth of `batch` same-shape matrices X + b*strideX -> Q + b*strideQ, all sharing the dust Z.
 * Each matrix gets exactly the bits spanqr_orth_f32 would give it, whatever the batch. */
int spanqr_orth_strided_f32(const float* X, long long ldx, long long strideX, float* Q, long long ldq,
                            long long strideQ, int K, int r, int batch, const float* Z, void* ws, size_t ws_bytes,
                            spanqr_stream_t stream);

/* the same with DEVICE arrays of per-matrix pointers dX[batch], dQ[batch] (leading dimension r for all; every
 * pointer 16-byte aligned) */
int spanqr_orth_batched_f32(const float* const* dX, float* const* dQ, int K, int r, int batch, const float* Z,
                            void* ws, size_t ws_bytes, spanqr_stream_t stream);

/* the same with HOST arrays hX[batch], hQ[batch] of device pointers (copied into kernel parameters, so no
 * host-to-device copy and no pinned memory is involved; leading dimension r for all) */
int spanqr_orth_ptrs_f32(const float* const* hX, float* const* hQ, int K, int r, int batch, const float* Z,
                         void* ws, size_t ws_bytes, spanqr_stream_t stream);

/*
 * orth of `batch` matrices of one width r and per-matrix heights K[b] (host arrays hX, hQ of device pointers with
 * leading dimension r, host array K, host array Z of per-matrix dust pointers: Z[b] is the dust of shape K[b] x r,
 * the same pointer for equal heights).  The workspace (spanqr_workspace_bytes_mixed) holds one batched call per
 * distinct height; the groups run one after another on `stream`, and each matrix gets the bits of a lone
 * spanqr_orth_f32 call.  No reference counterpart (the reference orthonormalises one layer at a time).
 */
int spanqr_workspace_bytes_mixed(const int* K, int r, int batch, size_t* bytes);
int spanqr_orth_mixed_f32(const float* const* hX, float* const* hQ, const int* K, int r, int batch,
                          const float* const* Z, void* ws, size_t ws_bytes, spanqr_stream_t stream);

/*
 * Q = borth(X) for r > 512 (orth.py:18-19 -> candidates/kbig.py:66-95, block Gram-Schmidt with reorthogonalisation
 * over 256-column blocks, every Cholesky 256 wide): X, Q fp32 row-major K x r (leading dimensions ldx, ldq; X and Q
 * must not overlap), r a multiple of 256 in [256, 16384], K >= r, K * 256 <= 2^31; Z the K x r dust of
 * kcholqr.py:83-89 (leading dimension r), block j using its columns j .. j + 255.  Each block is projected against the
 * finished ones twice (band Gram, W - P (P^T W) on the tensor cores, in place in Q), orthonormalised by the orth
 * sequence, projected and orthonormalised once more.  Stream-ordered, no host synchronisation, deterministic.  The
 * workspace (spanqr_workspace_bytes_borth) begins with a status word read by spanqr_read_status.
 */
int spanqr_workspace_bytes_borth(int K, int r, size_t* bytes);
int spanqr_borth_f32(const float* X, long long ldx, float* Q, long long ldq, int K, int r, const float* Z, void* ws,
                     size_t ws_bytes, spanqr_stream_t stream);

/*
 * orth of one shape as one CUDA graph (no reference counterpart; the reference launches kernel by kernel from Python,
 * candidates/kcholqr.py:92-112).  spanqr_orth_graph_create captures the whole kernel sequence of spanqr_orth_f32 for
 * shape K x r with leading dimensions ldx, ldq, the dust Z and the workspace ws (all baked into the graph; Z and ws must
 * stay valid and unchanged until the graph is destroyed) and instantiates it, on the current device, from outside any
 * stream capture; it enqueues nothing.  spanqr_orth_graph_launch replays it for Q = orth(X) on `stream`: only the
 * set-up kernel's X and Q arguments are replaced, so no copy of X or Q is made and every later kernel is launched as
 * captured; the bits equal spanqr_orth_f32's.  Launches of one graph share its workspace: issue them from one host
 * thread and keep them ordered on one stream (or serialise them), as with calls sharing a workspace.  The launch
 * returns SPANQR_ERR_ARG for other leading dimensions, a misaligned pointer or another current device.
 */
typedef struct spanqr_graph_st* spanqr_graph_t;
int spanqr_orth_graph_create(int K, int r, long long ldx, long long ldq, const float* Z, void* ws, size_t ws_bytes,
                             spanqr_graph_t* graph);
int spanqr_orth_graph_launch(spanqr_graph_t graph, const float* X, long long ldx, float* Q, long long ldq,
                             spanqr_stream_t stream);
int spanqr_orth_graph_destroy(spanqr_graph_t graph);

/*
 * orth of one matrix for callers that cannot allocate device memory: code running inside a CUDA stream capture
 * that must not add allocations, memory-capped sandboxes, or real-time loops that forbid cudaMalloc.  No
 * counterpart in the reference.  Instead of a caller workspace it uses a fixed scratch array of
 * SPANQR_NOALLOC_SCRATCH_BYTES (16 MiB) that lives in the library's device image: every GPU that loads the library
 * holds it until the process exits.  Shapes whose spanqr_workspace_bytes(K, r, 1) exceeds it return
 * SPANQR_ERR_TOO_LARGE.  The first call on each device looks up the array's device address (cudaGetSymbolAddress,
 * with that device current), so make that first call before any stream capture.  All calls share the one array:
 * calls that overlap on the GPU (other streams or threads) race and corrupt each other's results; serialise them.
 * Nothing is allocated or freed, by this library or by any library it calls.  The device address is cached per
 * device and per context: after a cudaDeviceReset the next call looks it up again (do that call outside a capture).
 */
#define SPANQR_NOALLOC_SCRATCH_BYTES (16u << 20)
int spanqr_orth_noalloc_f32(const float* X, long long ldx, float* Q, long long ldq, int K, int r, const float* Z,
                            spanqr_stream_t stream);

/*
 * The device status word of spanqr_orth_noalloc_f32's scratch array on the current device (the counterpart of
 * spanqr_read_status for that entry point, whose scratch the caller cannot address): 0 = the last no-allocation call
 * recorded no failure; otherwise its bounded device waits ran out and Q must not be used (SPANQR_ERR_DEVICE).  No
 * reference counterpart.  Synchronises `stream`; allocates nothing.
 */
int spanqr_noalloc_read_status(spanqr_stream_t stream, int* device_status);

/*
 * Component entry points (the reference's kernel modules), for tests and for callers that compose their own
 * recipe.  Each needs its own workspace of spanqr_workspace_bytes(K or n, n, 1) bytes.
 *
 * spanqr_gram_f32: G [n, n] = A^T A for A = s * Y (Y [K, n], leading dimension ldy), split-K with a compensated
 *   (Kahan) sum inside each split and an fp64 sum across splits; d_s: device pointer to the fp32 scale s, or NULL
 *   for s = 1.  G is written in full (both triangles, exactly symmetric).
 */
int spanqr_gram_f32(const float* Y, long long ldy, int K, int n, const float* d_s, float* G, void* ws,
                    size_t ws_bytes, spanqr_stream_t stream);

/*
 * spanqr_gram_mode_f32: the same G with the arithmetic of one of the orth sequence's Grams, so that each can be
 *   checked on its own: SPANQR_GRAM_ACCURATE (= spanqr_gram_f32), SPANQR_GRAM_PASS (the Gram of every Cholesky-QR
 *   pass and of the first polish step: the reference's gram_f in pass 1, tri.py:362-375, and its plain SGEMM
 *   Y.T @ Y, kcholqr.py:106), SPANQR_GRAM_POLISH (the last polish step's Gram: the reference's gram_split,
 *   kcholqr.py:20, tri.py:285-297).  Any other mode returns SPANQR_ERR_ARG.
 */
enum spanqr_gram_mode { SPANQR_GRAM_ACCURATE = 0, SPANQR_GRAM_PASS = 1, SPANQR_GRAM_POLISH = 2 };
int spanqr_gram_mode_f32(const float* Y, long long ldy, int K, int n, const float* d_s, int mode, float* G, void* ws,
                         size_t ws_bytes, spanqr_stream_t stream);

/*
 * spanqr_chol_f32: lower Cholesky factor of G [n, n] (lower triangle read, G left unchanged) with every pivot
 *   clamped from below at *d_tau (a NaN pivot also becomes tau): L [n, n] (zeros above the diagonal) and
 *   Li [n, 32], the inverses of L's 32 x 32 diagonal tiles stacked.  n a multiple of 32, at most 512.
 */
int spanqr_chol_f32(const float* G, int n, const float* d_tau, float* L, float* Li, void* ws, size_t ws_bytes,
                    spanqr_stream_t stream);

/*
 * spanqr_trsm_f32: Y = (s X + eps Z) L^-T with L, Li from spanqr_chol_f32; X [K, n] (ldx), Y [K, n] (ldy),
 *   Z [K, n] (leading dimension n) or NULL, d_s device pointer to s or NULL for s = 1.  Y may equal X (in place).
 */
int spanqr_trsm_f32(const float* X, long long ldx, const float* Z, const float* d_s, float eps, const float* L,
                    const float* Li, int K, int n, float* Y, long long ldy, void* ws, size_t ws_bytes,
                    spanqr_stream_t stream);

/*
 * Kernel timing (no reference counterpart; the reference stamps %globaltimer under CHOL_DEBUG, chol.cu:17-23).
 * mode 1: the orth entry points bracket every kernel they launch with CUDA events on the launching stream;
 * mode 2: they only count their launches (no events, nothing added to the streams); mode 0: off.
 * spanqr_timing_collect waits for the events, adds each kind's device time to ms[kind] and its kernel launches to
 * launches[kind] for kind < nkinds (k_ns_update counts its operand-image kernel too), and forgets them.  Kinds are numbered 0..spanqr_kernel_kinds()-1 (names from
 * spanqr_kernel_kind_name).  Timing state is per host thread.  A mode outside 0..2 returns SPANQR_ERR_ARG.
 */
int spanqr_timing_enable(int mode);
int spanqr_timing_collect(double* ms, long long* launches, int nkinds);
int spanqr_kernel_kinds(void);
const char* spanqr_kernel_kind_name(int kind);

/*
 * Reads the device status word of a workspace (0 = no failure recorded by the last call that used it).
 * This call synchronises `stream`.
 */
int spanqr_read_status(const void* ws, spanqr_stream_t stream, int* device_status);

/*
 * Self-test of the device timeout path (no reference counterpart; the reference's grid barrier spins without a
 * limit, candidates/cuk/chol.cu).  Zeroes the status word of `ws` (at least 256 bytes, 256-byte aligned) and
 * launches one warp that waits on an mbarrier phase for at most limit_ns (1 .. 2e9) nanoseconds; the phase
 * completes only if `arrive` is non-zero.  A wait that runs out sets bit 0x80 of the status word, read back with
 * spanqr_read_status (SPANQR_ERR_DEVICE), the same way a production kernel reports its own timeout bit (0x10 Gram,
 * 0x20 polish update, 0x40 solve).  The kernel returns either way and the context stays usable.
 */
int spanqr_selftest_timeout(void* ws, size_t ws_bytes, long long limit_ns, int arrive, spanqr_stream_t stream);

/*
 * Exchange slabs of orth_batched across the GPUs of one node (no reference counterpart: the reference is single-GPU;
 * these serve the all-gather of results when a batch is spread over 2-8 GPUs).  Every rank allocates one slab on its
 * current device (cudaMalloc) and exports it as a SPANQR_PEER_HANDLE_BYTES-byte CUDA IPC handle; every other rank of
 * the node, with its own device current, opens that handle into a pointer it can read (peer access enabled on first
 * use).  A handle cannot be opened by the process that exported it.  A rank's waves
 * write their Q into its own slab and every rank then pulls each owner's run from that owner's slab with
 * spanqr_peer_copy: one cudaMemcpyAsync, so the copy engines carry it over NVLink and no SM is taken from the waves
 * still computing.  The caller orders the copies after the owner's writes (a stream-ordered barrier across the ranks)
 * and closes every opened handle before the owner frees its slab.
 */
#define SPANQR_PEER_HANDLE_BYTES 64
int spanqr_peer_slab_alloc(size_t bytes, void** ptr, void* handle);
int spanqr_peer_slab_open(const void* handle, void** ptr);
int spanqr_peer_slab_close(void* ptr);
int spanqr_peer_slab_free(void* ptr);
int spanqr_peer_copy(void* dst, const void* src, size_t bytes, spanqr_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SPANQR_H */
