/*
 * bi.h -- C ABI of libbi.so, the batch-invariant GEMM and attention kernels for
 * NVIDIA B200 (sm_100a).
 *
 * Every entry point takes plain device pointers, element counts and a CUDA stream
 * handle (cudaStream_t passed as void*).  Nothing here allocates device memory, no
 * call synchronises the stream, and no call aborts: each returns a bi_status.
 * Work is enqueued asynchronously on `stream` and is safe to capture in a CUDA
 * graph.
 *
 * The reference library (mlx-batch-invariant 0.2.0) has no C ABI of its own: its
 * kernels are Metal source strings launched by MLX from Python.  Each entry point
 * below replaces the Python-level operator named beside it; the Python package
 * mlx_batch_invariant_b200 binds them with ctypes and keeps the reference's
 * signatures, argument meaning and errors.
 *
 * Invariance contract: for a given (K, N, dtype, layout) the GEMM uses one tile
 * shape and one K order whatever M is, and the attention kernel folds keys in one
 * fixed order whatever B, H, qL are; so any output row's bits do not depend on the
 * other rows computed with it.
 */
#ifndef BI_H_
#define BI_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types.  The values are part of the ABI. */
typedef enum {
  BI_F32 = 0,
  BI_F16 = 1,
  BI_BF16 = 2
} bi_dtype;

/* Status codes: 0 on success, negative on error. */
typedef enum {
  BI_OK = 0,
  BI_ERR_INVALID = -1,       /* bad shape, stride, pointer or argument          */
  BI_ERR_UNSUPPORTED = -2,   /* valid request this build has no kernel for      */
  BI_ERR_MISALIGNED = -3,    /* pointer or stride breaks the 16-byte rule       */
  BI_ERR_CUDA = -4,          /* a CUDA runtime call failed (see message)        */
  BI_ERR_TIMEOUT = -5,       /* a bounded device-side wait gave up (device flag) */
  BI_ERR_NO_DEVICE = -6      /* no CUDA device / not an sm_100 device            */
} bi_status;

/* Routes a GEMM can take (see bi_gemm_route). */
typedef enum {
  BI_ROUTE_TCGEN05 = 0,      /* tcgen05/TMEM tensor-core kernel fed by TMA      */
  BI_ROUTE_SIMT = 1          /* CUDA-core fp32 FMA kernel, sequential K         */
} bi_route;

/*
 * out[m, n] = round_T( alpha * sum_k a[m, k] * B[k, n]  (+ beta * bias[n]) )
 *
 * Replaces mlx_batch_invariant/_gemm.py:_gemm (and through it matmul :225-227,
 * addmm :230-232, linear :235-240 of the reference, whose kernel is the MSL
 * string bi_gemm at _gemm.py:29-130).
 *
 *   a      (M, K) row-major, row stride lda elements.
 *   b      b_is_nk = 1: (N, K) row-major (the nn.Linear weight layout), stride ldb.
 *          b_is_nk = 0: (K, N) row-major, stride ldb.
 *   bias   nullable; (N,) contiguous.  When null, alpha and beta are ignored and the
 *          accumulator is rounded as is (reference: HAS_BIAS = 0).
 *   out    (M, N) row-major, row stride ldo elements, same dtype as a and b.
 *
 * The sum is accumulated in fp32 over k in one fixed order that depends only on
 * (K, dtype), with no split-K, no atomics; the bias is added to the fp32 value
 * (v = alpha*acc, then v + beta*bias, each rounded to fp32) before the single
 * rounding to the output type.  M = 0 or N = 0 is a no-op; K = 0 gives the bias
 * term alone.
 */
int bi_gemm(const void* a, int64_t lda, const void* b, int64_t ldb,
            const void* bias, void* out, int64_t ldo,
            int64_t M, int64_t N, int64_t K, int b_is_nk,
            float alpha, float beta, int dtype, void* stream);

/*
 * float32 bi_gemm on the tensor cores: the same contract as bi_gemm with dtype BI_F32,
 * run as three tf32 products per K step (tcgen05.mma kind::tf32: a_big*b_big +
 * a_big*b_small + a_small*b_big, x = big + small exactly, big = x with its low 13
 * mantissa bits cleared) with fp32 accumulation of each 256-deep K chunk on the
 * tensor cores and the chunk sums added in K order in fp32 (round to nearest); one
 * 256 x 256 pair tile and K order for every M, so rows are batch-invariant.  Within the reference's float32
 * accuracy bar against float64 (mlx_batch_invariant tests/test_invariance.py:114-127),
 * not bit-equal to bi_gemm's CUDA-core fp32 route.  No counterpart in the reference
 * (whose fp32 path is the same bi_gemm kernel).  Needs K % 4 == 0 (and N % 4 == 0 for
 * a (K, N) b), 16-byte aligned a / b and row strides that are multiples of 4 elements;
 * else BI_ERR_UNSUPPORTED / BI_ERR_MISALIGNED.
 */
int bi_gemm_tf32x3(const void* a, int64_t lda, const void* b, int64_t ldb,
                   const void* bias, void* out, int64_t ldo,
                   int64_t M, int64_t N, int64_t K, int b_is_nk,
                   float alpha, float beta, void* stream);

/*
 * The kernel route and CTA tile bi_gemm uses for (dtype, K, N, layout).  The result
 * never depends on M; this is the library's analogue of the reference's public
 * TILE constant (_gemm.py:27).  Any out-pointer may be null.
 */
int bi_gemm_route(int dtype, int64_t K, int64_t N, int b_is_nk,
                  int* route, int* bm, int* bn, int* bk);

/*
 * out[b, h, s, :] = softmax(scale * q[b, h, s, :] . k[b, kvh, i, :] + mask) . v
 *
 * Replaces mlx_batch_invariant/_attention.py:scaled_dot_product_attention
 * (:205-250) and its MSL kernel bi_sdpa (:32-149).
 *
 *   q      (B, H, qL, D) with element strides q_strides[0..2] for b, h, s; the last
 *          dimension contiguous.
 *   k, v   (B, Hkv, N, D) and (B, Hkv, N, V); strides k_strides / v_strides for b
 *          and h; each head's (N, D) block must be row-contiguous.
 *   mask   mask_mode 0: none.  1: causal, query s sees keys i <= causal_offset + s
 *          (the reference's bottom-right rule is causal_offset = N - qL).
 *          2: additive mask in the q dtype, element strides mask_strides[0..2] for
 *          (b, h, s) (0 to broadcast), last dimension contiguous; a key whose mask
 *          value is <= -3e38 (i.e. -inf) is skipped, not added.
 *   sinks  nullable; (H,) in the q dtype, one extra logit per query head
 *          (reference _attention.py:80-86).
 *   out    (B, H, qL, V) with element strides out_strides[0..2], last dim contiguous.
 *
 * H % Hkv == 0; D and V multiples of 32, D, V <= 640 for fp16 / bf16 and D, V <= 384,
 * D + V <= 768 for fp32 (else BI_ERR_UNSUPPORTED); D may differ from V.  Each (query row,
 * head) is reduced by one CTA over all N keys in 32 fixed strides (key i folds into
 * partial i % 32) with an fp32 online softmax and a fixed combine; there is no
 * split-KV and no route that depends on qL, B or N.  A row with no visible key
 * returns zeros.
 */
int bi_sdpa(const void* q, const int64_t q_strides[3],
            const void* k, const int64_t k_strides[2],
            const void* v, const int64_t v_strides[2],
            const void* mask, const int64_t mask_strides[3], int mask_mode,
            int64_t causal_offset, const void* sinks, float scale,
            int64_t B, int64_t H, int64_t Hkv, int64_t qL, int64_t N,
            int64_t D, int64_t V, int dtype,
            void* out, const int64_t out_strides[3], void* stream);

/*
 * ---------------------------------------------------------------------------
 * Multi-GPU: the column-parallel GEMM with its all-gather fused into the epilogue.
 *
 * No reference counterpart (the reference is single-device); this is the exchange
 * step of the column-parallel plan in which rank s owns output columns
 * [cols[s], cols[s+1]).  Instead of a separate all-gather, every CTA stores each
 * finished output tile into this rank's output and, through NVLink peer mappings,
 * into every other rank's staging area as part of one dense (M, N_local) block; ranks
 * then exchange epoch flags (bounded waits) and each copies the blocks it received
 * into its output.  The bits are those of bi_gemm on the full weight.
 * ---------------------------------------------------------------------------
 */

/* Maximum number of ranks bi_gemm_allgather / bi_peer_barrier take. */
#define BI_MAX_PEERS 8

/* Bytes of the flag block each rank's exchange buffer must end with. */
#define BI_PEER_FLAG_BYTES 256

/* Allocates `bytes` of device memory that peers may map (zero-filled), and writes
 * its CUDA IPC handle (64 bytes) to ipc_handle.  Set-up call, not on the hot path. */
int bi_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle);
/* Maps a peer's buffer from its IPC handle (another process's bi_peer_alloc). */
int bi_peer_open(const void* ipc_handle, void** ptr);
/* Unmaps a buffer mapped with bi_peer_open. */
int bi_peer_close(void* ptr);
/* Frees a buffer from bi_peer_alloc (after every peer has unmapped it). */
int bi_peer_free(void* ptr);

/* Stream-ordered barrier over `world` ranks: rank `rank` posts `epoch` to every
 * rank's flag block and waits (bounded) until every rank has posted it to its own.
 * flags[r] is rank r's flag block (BI_PEER_FLAG_BYTES), mapped in this process.
 *
 * Epochs (here and in bi_gemm_allgather*): either every call on a flag block passes
 * a value larger than any earlier call's, or every call passes 0 and the block counts
 * its calls itself (a word in the block, advanced on the device by each call's entry
 * barrier).  Use 0 for calls captured in a CUDA graph, whose replays repeat their
 * arguments.  Ranks must make the same calls in the same order either way. */
int bi_peer_barrier(void* const* flags, int rank, int world, uint32_t epoch, void* stream);

/*
 * Column-parallel y = x . w^T (+ bias) with the all-gather fused into the epilogue.
 *   a          (M, K) activations, replicated on every rank.
 *   b          this rank's weight shard: (N_local, K) if b_is_nk, else (K, N_local),
 *              N_local = cols[rank+1] - cols[rank].
 *   bias       nullable; this rank's (N_local,) slice.
 *   out        this rank's (M, ldo) output, any device memory of this rank (it is only
 *              written locally); ldo >= cols[world], a multiple of 8.
 *   stages[r]  rank r's staging area mapped here (stages[rank] is local): at least
 *              M * cols[world] elements; rank s writes its block (M, N_s) row-major at
 *              element offset M * cols[s] of every other rank's area.
 *   cols       world + 1 column bounds: cols[0] = 0, nondecreasing, multiples of 8.
 *   flags[r]   rank r's flag block.  epoch: see bi_peer_barrier (0 = counted on the
 *              device, for graph capture).
 * On return (stream order) `out` holds all cols[world] columns.  Calls an entry barrier
 * first, so no peer writes a staging area its owner may still read.  Same arithmetic,
 * tile and route rules as bi_gemm.
 */
int bi_gemm_allgather(const void* a, int64_t lda, const void* b, int64_t ldb,
                      const void* bias, void* out, int64_t ldo,
                      void* const* stages, const int64_t* cols,
                      int64_t M, int64_t K, int b_is_nk,
                      float alpha, float beta, int dtype,
                      void* const* flags, int rank, int world, uint32_t epoch,
                      void* stream);

/*
 * bi_gemm_allgather in two halves, so the local copy of the received blocks can run
 * on another stream, under the next call's GEMM (no reference counterpart).
 *
 * bi_gemm_allgather_deferred takes bi_gemm_allgather's arguments and enqueues the
 * entry barrier and the GEMM with its peer stores and exit barrier: on return (stream
 * order) `out` holds this rank's own columns and every peer's block has landed in
 * this rank's staging area.  bi_gather_unpack then copies those blocks into the other
 * columns of `out` -- on `stream` after the GEMM (order it with an event when it is
 * another stream).  Until that copy has run, this rank must make no further call on
 * the same staging area (its entry barrier would let the peers overwrite it).
 */
int bi_gemm_allgather_deferred(const void* a, int64_t lda, const void* b, int64_t ldb,
                               const void* bias, void* out, int64_t ldo,
                               void* const* stages, const int64_t* cols,
                               int64_t M, int64_t K, int b_is_nk,
                               float alpha, float beta, int dtype,
                               void* const* flags, int rank, int world, uint32_t epoch,
                               void* stream);
/* Copies rank s's dense (M, cols[s+1] - cols[s]) block, stored at element offset
 * M * cols[s] of stages[rank], into columns [cols[s], cols[s+1]) of `out` (row stride
 * ldo) for every s != rank.  Only stages[rank] is read. */
int bi_gather_unpack(void* out, int64_t ldo, void* const* stages, const int64_t* cols,
                     int64_t M, int rank, int world, int dtype, void* stream);

/*
 * bi_gemm_allgather for callers that may not allocate device memory.  No counterpart
 * in the reference (which is single-device).
 *
 * bi_gemm_allgather needs a flag block per rank from bi_peer_alloc, which calls
 * cudaMalloc.  Some callers cannot do that: a serving process whose device memory is
 * all handed out up front by its own allocator (weights, KV cache, activation arena)
 * and which must not have a library take memory behind that allocator's back, or a
 * host program that only ever passes buffers it owns.  This entry point allocates
 * nothing and calls no cudaMalloc, cudaFree or other allocating routine.  The fused
 * GEMM's own scratch -- its CTA-completion counter and the call count -- lives in a
 * 256-byte file-scope device array inside libbi.so (one copy per GPU that loads the
 * library, held until the process exits, touched only by kernels on that GPU); the
 * flags the ranks post to one another sit at the head of the exchange areas the
 * caller passes, which the peers must reach anyway.
 *
 *   stages[r]   rank r's exchange area, mapped here: BI_PEER_FLAG_BYTES bytes of
 *               flags (zero them once, before the first call; later calls use what
 *               earlier ones left), then the staging area of bi_gemm_allgather
 *               (M * cols[world] elements) -- at least BI_PEER_FLAG_BYTES + 2 * M *
 *               cols[world] bytes, 16-byte aligned.
 *   devices[r]  the CUDA device ordinal rank r runs on, all in THIS process (one
 *               process drives every rank), one rank per device: a repeated ordinal
 *               is rejected (BI_ERR_INVALID), and so is a call whose devices[rank]
 *               is not the current device.  The call enables peer access from the
 *               current device to every other rank's device (already enabled counts
 *               as success) and returns BI_ERR_UNSUPPORTED where the hardware has
 *               none.
 *   world       at most BI_MAX_PEERS; larger values are rejected (BI_ERR_INVALID)
 *               because the flag block holds flags for BI_MAX_PEERS ranks.
 * Everything else is as in bi_gemm_allgather.
 *
 * The first call on a device looks up its copy of the array with that device current
 * (cudaGetSymbolAddress) and caches the address; make that first call before any
 * stream capture.  All calls on a device share the array, which keeps the last call's
 * contents: each call clears the CTA counter on `stream` before use, and `epoch` must
 * exceed the epoch of every earlier call on the same exchange areas (or be 0 on every
 * call on the device: the array then counts the calls itself).  Calls whose work
 * overlaps on the GPU (different streams, or different rank groups sharing a device)
 * race on the array.
 */
int bi_gemm_allgather_static(const void* a, int64_t lda, const void* b, int64_t ldb,
                             const void* bias, void* out, int64_t ldo,
                             void* const* stages, const int64_t* cols,
                             int64_t M, int64_t K, int b_is_nk,
                             float alpha, float beta, int dtype, const int* devices,
                             int rank, int world, uint32_t epoch, void* stream);

/*
 * ---------------------------------------------------------------------------
 * Elementwise steps of the decoder harness, fused.  No reference counterpart: the
 * reference's harness (bench/bench.py:108-159) runs its framework's own ops.  Each
 * output element is computed from its own inputs with the fp32 operations of the
 * expression named, each rounded, so both are batch-invariant.
 * ---------------------------------------------------------------------------
 */

/* Rotary embedding (rotate-half) of the q and k heads of a fused q/k/v projection,
 * with the KV-cache write:
 *   qkv    (B, L, (hq + 2 hk) * hd) contiguous: hq query heads, then hk key heads, then
 *          hk value heads, each hd wide.
 *   row l of batch b sits at position p = (pos ? *pos : p0) + l (pos: device pointer,
 *          so a captured graph can advance it);
 *   q_out  (B, hq, L, hd) contiguous <- rotated q;
 *   k_cache[b, h, p, :] <- rotated k;  v_cache[b, h, p, :] <- v   (cache_strides =
 *          element strides of batch, head and position; the last dim contiguous).
 *   Rotation with c = cos_tab[p, i], s = sin_tab[p, i] (fp32, (positions, hd/2)):
 *   out[i] = x[i]*c - x[i+hd/2]*s,  out[i+hd/2] = x[i+hd/2]*c + x[i]*s.
 *   n_pos  the positions both tables and both caches hold.  With pos == NULL the call
 *          checks p0 + L <= n_pos (else BI_ERR_INVALID).  With a device `pos` the kernel
 *          writes no row whose position falls outside [0, n_pos) and records site 1,
 *          reason 2 (tagged bit 17) in the device error word (bi_device_error). */
int bi_rope_kv(const void* qkv, int64_t B, int64_t L, int64_t hq, int64_t hk, int64_t hd,
               const float* cos_tab, const float* sin_tab, int64_t p0, const int64_t* pos,
               int64_t n_pos, void* q_out, void* k_cache, void* v_cache,
               const int64_t cache_strides[3], int dtype, void* stream);

/* SwiGLU: gu (M, 2I) holds [gate | up] per row; out (M, I) = silu(gate) * up with silu
 * rounded to the storage type before the product, as silu(g) * u in two steps. */
int bi_swiglu(const void* gu, void* out, int64_t M, int64_t I, int dtype, void* stream);

/* Static description of a status code. */
const char* bi_status_string(int status);

/* Detail of the last host-side error on the calling thread ("" if none). */
const char* bi_last_error(void);

/*
 * Reads and (if clear != 0) resets the device-side error word of the current
 * device.  Kernels set it, instead of hanging, when a bounded wait gives up.
 * Synchronises the device.  Returns 0 when no kernel reported an error, else the
 * code a kernel stored (site << 8 | reason).
 */
int bi_device_error(int clear);

/* Library version as major*10000 + minor*100 + patch. */
int bi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* BI_H_ */
