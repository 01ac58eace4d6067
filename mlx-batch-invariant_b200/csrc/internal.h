// Host-side interfaces between the translation units of libbi.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bi.h"

namespace bi {

struct GemmArgs {
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  const void* bias;  // nullable
  void* out;
  int64_t ldo;
  int64_t M, N, K;
  int b_is_nk;
  float alpha, beta;
  int dtype;
};

// Column-parallel GEMM with the all-gather fused into the epilogue.  Rank s owns the
// global columns [cols[s], cols[s+1]).  Its finished tiles go to its own output
// directly and, over NVLink, into every other rank's staging area as one dense
// (M, cols[s+1] - cols[s]) row-major block at element offset M * cols[s]; each rank then
// copies the blocks it received into its output (gather_unpack_kernel).
struct GatherArgs {
  void* stages[BI_MAX_PEERS];     // every rank's staging area, mapped here
  uint32_t* flags[BI_MAX_PEERS];  // every rank's flag block, mapped here
  uint32_t* local;                // this rank's counters (its own device's memory only)
  int64_t cols[BI_MAX_PEERS + 1]; // column partition: rank s owns [cols[s], cols[s+1])
  int rank, world;
  uint32_t epoch;
};

// Flag block layout (32-bit words): [0, 8) exit flags posted by rank r, [8, 16) entry
// flags posted by rank r -- written by every rank -- and, in the block `local` points
// at, [16] the CTA-completion counter of the local GEMM and [17] the call count (the
// epoch of calls made with epoch 0) -- touched by this rank alone.  bi_gemm_allgather
// keeps both halves in one block (local = flags[rank]); bi_gemm_allgather_static keeps
// the counters in the library's own per-device array and the flags in the callers'
// exchange areas, so no device touches another device's copy of that array.
constexpr int kFlagExit = 0;
constexpr int kFlagEntry = BI_MAX_PEERS;
constexpr int kFlagCounter = 2 * BI_MAX_PEERS;
constexpr int kFlagEpoch = 2 * BI_MAX_PEERS + 1;

struct SdpaArgs {
  const void* q;
  int64_t qs[3];
  const void* k;
  int64_t ks[2];
  const void* v;
  int64_t vs[2];
  const void* mask;
  int64_t ms[3];
  int mask_mode;
  int64_t causal_offset;
  const void* sinks;
  float scale;
  int64_t B, H, Hkv, qL, N, D, V;
  int dtype;
  void* out;
  int64_t os[3];
};

// Fixed tile constants of the tensor-core route (bf16 / fp16): 128 rows per CTA (a
// 256 x 256 pair tile) and a 64-deep K block.
constexpr int kTcBM = 128;
constexpr int kTcBN = 256;
constexpr int kTcBK = 64;
// Fixed tile constants of the CUDA-core route.
constexpr int kSimtBM = 128;
constexpr int kSimtBN = 128;
constexpr int kSimtBK = 8;

// Tiled TMA descriptor over 16-bit data of `rank` dims (innermost first), strides in
// bytes for dims 1.., 128-byte swizzle, zero fill outside.  Defined with the GEMM.
int encode_tiled16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides, const uint32_t* box, int dtype);

// Decoder-harness elementwise steps (harness.cu).
struct RopeArgs {
  const void* qkv;         // (B, L, (hq + 2 hk) * hd): q heads, k heads, v heads
  int64_t B, L, hq, hk, hd;
  const float* cos_tab;    // (positions, hd / 2)
  const float* sin_tab;
  int64_t p0;
  const int64_t* pos;      // nullable: row l sits at position (pos ? *pos : p0) + l
  int64_t n_pos;           // positions the tables and the caches hold
  void* q_out;             // (B, hq, L, hd)
  void* k_cache;
  void* v_cache;
  int64_t cs0, cs1, cs2;   // cache strides (elements) of batch, head, position
};
int launch_rope_kv(const RopeArgs& a, int dtype, cudaStream_t stream);
int launch_swiglu(const void* gu, void* out, int64_t M, int64_t I, int dtype,
                  cudaStream_t stream);

int launch_gemm_tc(const GemmArgs& g, cudaStream_t stream);
// g.out points at column cols[rank] of the output whose first column is out_base.
// unpack = false leaves the peers' blocks in this rank's staging area (launch
// launch_gather_unpack later, possibly on another stream).
int launch_gemm_tc_allgather(const GemmArgs& g, const GatherArgs& x, void* out_base,
                             cudaStream_t stream, bool unpack);
int launch_gather_unpack(const GatherArgs& x, void* out_base, int64_t ldo, int64_t M,
                         cudaStream_t stream);
int launch_peer_barrier(const GatherArgs& x, cudaStream_t stream);
int static_flag_block(int device, void** out);
int launch_gemm_simt(const GemmArgs& g, cudaStream_t stream);
int launch_gemm_tf32x3(const GemmArgs& g, cudaStream_t stream);
int launch_sdpa(const SdpaArgs& s, cudaStream_t stream);

// Device error words, one per translation unit; read and optionally clear.
unsigned read_error_gemm_tc(bool clear);
unsigned read_error_sdpa(bool clear);
unsigned read_error_harness(bool clear);
unsigned read_error_tf32x3(bool clear);

// Per-thread message for bi_last_error().
int set_error(int status, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);

// Current device's SM count and compute capability (cached per device).
int device_sm_count();
int device_cc_major();

}  // namespace bi
