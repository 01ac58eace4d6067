// Batch-invariant GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), fed by
// TMA, for fp16 and bf16 inputs with fp32 accumulation.
//
// Invariance argument (the property mlx_batch_invariant/_gemm.py:1-24 states for
// its Metal kernel): every output element is produced by one CTA pair that owns the
// whole K reduction.  The tile (256 x 256 per pair), the K block (64) and the UMMA
// instruction (2-SM, M=256, N=256, K=16) are compile-time constants, so element
// (m, n) is always accumulated as the same sequence of K=16 tensor-core steps, k
// ascending, into an fp32 TMEM accumulator -- for every M, every row position in the
// tile and every column shard.  There is no split-K, no stream-K and no atomic.
// Which pair takes which tile (the persistent schedule below) changes with M; the
// arithmetic per element does not.
//
// Structure: clusters of two CTAs (a "pair", one per SM) run persistently.  Each CTA
// loads its own 128 rows of the A tile and its own 128 columns of the B tile with TMA
// into a 6-stage ring (no multicast); the leader CTA's MMA thread issues 2-SM UMMAs
// (tcgen05.mma.cta_group::2) that read both CTAs' shared memory and write rows
// 0-127 of the fp32 accumulator to the leader's TMEM and rows 128-255 to the peer's.
//   warp 0      TMA producer (both CTAs); the leader's full barrier counts both
//               CTAs' bytes.
//   warp 1      TMEM allocator (both CTAs) and, in the leader, the UMMA issuer; two
//               256-column accumulator buffers so tile i's epilogue overlaps tile
//               i+1's main loop.  Commits multicast to both CTAs' barriers.
//   warps 2..5  epilogue (both CTAs): tcgen05.ld of the CTA's 128 rows, alpha/bias in
//               fp32, one rounding to the output type, vector stores; they release
//               the accumulator on the leader's barrier.
// Every mbarrier wait is bounded; a wait that gives up raises the device error word
// and the CTA drains what it started, frees TMEM and exits.
//
// Fused all-gather (GATHER = true, column-parallel over ranks): the epilogue stores
// each finished block into this rank's output and, through NVLink peer mappings, into
// every other rank's staging area, where this rank's shard is one dense (M, N_local)
// row-major block.  A full 32 x 128 block leaves the staging buffer by TMA stores (one
// thread issues them, one box per 64 columns per destination; no multicast), so the
// epilogue warps go back to the accumulator while the copy engine feeds the links;
// ragged edges use plain 16-byte or element stores.  A dense block keeps the
// span of remote addresses in flight small: stores scattered straight into 8 peers'
// row-major outputs (rows N_total apart) ran 10x slower than the link at 8 GPUs.
// Each storing thread fences at system scope; the last CTA of the grid (a counter in
// the local flag block) then posts the call's epoch to every rank's exit flag with a
// release store and waits, bounded, until every rank has posted it.  A second kernel
// (gather_unpack_kernel) then copies the received blocks into the output.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace bi {

// Scratch of bi_gemm_allgather_static: the local GEMM's CTA-completion counter and the
// call count, kept in a file-scope device array instead of caller-allocated memory.
// Every device that loads this library holds its own 256-byte copy until the process
// exits; all calls on a device share it, and only kernels on that device touch it.
static __device__ __align__(256) uint32_t g_static_flag_block[BI_PEER_FLAG_BYTES / 4];

namespace tc {

constexpr int BM = kTcBM;    // rows per CTA (the pair covers 2*BM)
constexpr int BK = kTcBK;    // 64 x 2 bytes = one 128-byte swizzle row
constexpr int UMMA_K = 16;
constexpr int ACC_BUFS = 2;
constexpr int NUM_THREADS = 192;
constexpr int EPI_WARPS = 4;
// Epilogue staging: each epilogue warp turns 32 rows x 128 columns of finished outputs
// around in shared memory so a store instruction writes 256 contiguous bytes of a row.
constexpr int EPI_COLS = 128;
constexpr int EPI_STAGE_BYTES = 32 * EPI_COLS * 2;  // per warp, 16-bit outputs

// The shared-memory ring that feeds the UMMAs.  It decides how many rows of A each
// stage holds and how many stages are in flight -- never the tile, the instruction or
// the K order.
//   Wide ring  every CTA loads its 128 rows of A; 6 stages of 16 + 16 KiB.
//   Thin ring  M <= 16: only rows 0-15 of the pair tile exist, so CTA 0 loads a
//              16-row A box and CTA 1 none; the freed memory holds 10 stages, keeping
//              160 KiB of W in flight per SM (decode is bound by streaming W).
//              The UMMA still reads 128 rows per CTA: rows past the box hold whatever
//              the shared memory held, which only reaches output rows >= 16 (>= M),
//              and those are never stored.
template <int A_ROWS_, int STAGES_>
struct RingCfg {
  static constexpr int A_ROWS = A_ROWS_;
  static constexpr int STAGES = STAGES_;
  static constexpr int BN = kTcBN;              // columns per pair tile
  static constexpr int BN_CTA = BN / 2;         // B columns each CTA loads
  static constexpr int TMEM_COLS = ACC_BUFS * BN;
  static constexpr bool THIN = A_ROWS_ < BM;
  static constexpr int A_STAGE_BYTES = A_ROWS * BK * 2;
  static constexpr int B_STAGE_BYTES = BN_CTA * BK * 2;
  static constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
  static constexpr int NUM_BARRIERS = 2 * STAGES + 2 * ACC_BUFS + 1;
  static constexpr int SMEM_BYTES = 1024 /* alignment slack */ + STAGES * STAGE_BYTES +
                                    EPI_WARPS * EPI_STAGE_BYTES + NUM_BARRIERS * 8 + 16;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory above the per-CTA limit");
  static_assert(A_STAGE_BYTES % 1024 == 0 && B_STAGE_BYTES % 1024 == 0,
                "stages must keep 1 KiB swizzle alignment");
};
using WideRing = RingCfg<BM, 6>;
using ThinRing = RingCfg<16, 10>;
constexpr int THIN_MAX_M = ThinRing::A_ROWS;

constexpr uint16_t PAIR_MASK = 0x3;

// Error sites (code = site << 8 | reason).
enum : unsigned {
  kSiteProducer = 1,
  kSiteMma = 2,
  kSiteEpilogue = 3,
  kSiteDrain = 4,
  kSitePeerExit = 5,
  kSitePeerEntry = 6
};

__device__ unsigned g_error_word = 0;

struct Params {
  const void* bias;
  void* out;
  int64_t ldo;
  int M, N, K;
  float alpha, beta;
  int has_bias;
  int tiles_m, tiles_n, num_tiles;
  int group_m;    // pair-tiles of M that consecutive tile indices sweep (L2 reuse of W)
  GatherArgs gx;  // used when GATHER
  int tma_store;  // GATHER: full staged blocks leave by TMA stores through StoreMaps
};

// GATHER: where this rank's block goes.  m[d] is rank d's copy of it -- the output
// itself at d == rank, rank d's staging block otherwise -- as a (N_local, M) 16-bit
// tensor with a 64 x 32 box and the 128-byte swizzle of the staging buffer.
struct alignas(64) StoreMaps {
  CUtensorMap m[BI_MAX_PEERS];
};

// Byte offset of 16-byte chunk u (0..15, 8 columns each) of row r (0..31) in an
// epilogue warp's staging buffer.  Plain GEMM: 256-byte rows, chunk u at u ^ (r & 15).
// GATHER: two 64-column halves of 32 rows x 128 bytes, each in the TMA 128-byte
// swizzle (chunk u & 7 of row r at (u & 7) ^ (r & 7)), the layout a TMA store reads.
// Both keep a warp's row-per-lane writes and row-pair reads free of bank conflicts.
template <bool GATHER>
__device__ __forceinline__ int stage_off(int r, int u) {
  if constexpr (GATHER) return ((u >> 3) << 12) + r * 128 + (((u & 7) ^ (r & 7)) << 4);
  return r * (EPI_COLS * 2) + ((u ^ (r & 15)) << 4);
}

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int group_m,
                                            int& tm, int& tn) {
  const int per_group = group_m * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * group_m;
  const int rows = min(tiles_m - first_m, group_m);
  const int in_group = tile - group * per_group;
  tm = first_m + in_group % rows;
  tn = in_group / rows;
}

// The epoch of the current call: the explicit one, or (epoch 0) the count the call's
// entry barrier stored in the local flag block.
__device__ __forceinline__ uint32_t call_epoch(const GatherArgs& x) {
  return x.epoch != 0 ? x.epoch
                      : *reinterpret_cast<volatile uint32_t*>(x.local + kFlagEpoch);
}

template <typename T, bool B_NK, bool GATHER, typename R>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, const Params p,
                   const __grid_constant__ StoreMaps smap) {
  constexpr int STAGES = R::STAGES;
  constexpr int BN = R::BN;
  constexpr int BN_CTA = R::BN_CTA;
  constexpr int TMEM_COLS = R::TMEM_COLS;
  constexpr int B_STAGE_BYTES = R::B_STAGE_BYTES;
  constexpr int A_STAGE_BYTES = R::A_STAGE_BYTES;
  constexpr int STAGE_BYTES = R::STAGE_BYTES;
  constexpr int NUM_BARRIERS = R::NUM_BARRIERS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  uint8_t* epi_stage = smem + STAGES * STAGE_BYTES;  // EPI_WARPS x EPI_STAGE_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + EPI_WARPS * EPI_STAGE_BYTES);
  uint64_t* full = bars;                              // used in the leader
  uint64_t* empty = bars + STAGES;                    // both CTAs
  uint64_t* tfull = bars + 2 * STAGES;                // both CTAs
  uint64_t* tempty = bars + 2 * STAGES + ACC_BUFS;    // used in the leader
  uint64_t* mma_done = bars + 2 * STAGES + 2 * ACC_BUFS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARRIERS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader, 1 = peer
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < ACC_BUFS; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * EPI_WARPS);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (p.K + BK - 1) / BK;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      const uint32_t full_leader0 = map_to_cta(smem_u32(&full[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs) {
        int tm, tn;
        tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          // the leader's barrier counts both CTAs' bytes (a thin ring: one A box)
          if (leader) {
            mbar_arrive_expect_tx(&full[stage],
                                  (R::THIN ? 1 : 2) * A_STAGE_BYTES + 2 * B_STAGE_BYTES);
          }
          const uint32_t bar = full_leader0 + stage * 8;
          if (!R::THIN || leader) {
            tma_load_2d_pair(sA + stage * A_STAGE_BYTES, &tmap_a, bar, kb * BK,
                             tm * 2 * BM + static_cast<int>(rank) * BM);
          }
          uint8_t* dstB = sB + stage * B_STAGE_BYTES;
          const int n0 = tn * BN + static_cast<int>(rank) * BN_CTA;
          if (B_NK) {
            tma_load_2d_pair(dstB, &tmap_b, bar, kb * BK, n0);
          } else {
            // (K, N) row-major B: two 64-column slabs, each 64 k-rows of 128 bytes.
#pragma unroll
            for (int j = 0; j < BN_CTA / 64; ++j) {
              tma_load_2d_pair(dstB + j * (64 * BK * 2), &tmap_b, bar, n0 + j * 64, kb * BK);
            }
          }
          issued_any = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        record_error(&g_error_word, (kSiteProducer << 8) | kErrReasonTimeout);
        // Drain: the fills complete on the leader's barriers; give them a bounded
        // moment to land before this CTA's shared memory is released.
        if (issued_any) sleep_ns(200000);
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer (leader only) ----------------
    if (leader && lane == 0) {
      constexpr uint32_t fmt = (dtype_of<T>::value == 2) ? 1u : 0u;
      constexpr uint32_t idesc = umma_idesc_f16(fmt, B_NK ? 0u : 1u, 2 * BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[buf], acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // K-major, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart;
            // the K=16 step moves 32 bytes along the row.
            const uint64_t adesc = umma_smem_desc(a_base + k * UMMA_K * 2, 16, 1024, 2);
            uint64_t bdesc;
            if (B_NK) {
              bdesc = umma_smem_desc(b_base + k * UMMA_K * 2, 16, 1024, 2);
            } else {
              // MN-major, 128-byte swizzle: 64-column slabs 8 KiB apart (LBO), 8-k-row
              // groups 1024 B apart (SBO); the K=16 step moves 16 rows = 2048 B.
              bdesc = umma_smem_desc(b_base + k * UMMA_K * 128, 64 * BK * 2, 1024, 2);
            }
            umma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], PAIR_MASK);  // frees the stage in both CTAs
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[buf], PAIR_MASK);  // accumulator ready in both CTAs
      }
      if (!ok) {
        *abort_flag = 1;
        record_error(&g_error_word, (kSiteMma << 8) | kErrReasonTimeout);
      }
      // Whatever happened, wait until every MMA this thread issued has finished
      // before either CTA releases TMEM and shared memory.
      umma_commit_pair(mma_done, 0x1);
      if (!mbar_wait(mma_done, 0, nullptr)) {
        record_error(&g_error_word, (kSiteDrain << 8) | kErrReasonTimeout);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may access: 32*quarter..+31
    const T* bias = static_cast<const T*>(p.bias);
    T* out = static_cast<T*>(p.out);
    const bool vec_ok = (p.ldo % 8 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
    // GATHER: element offset of this rank's (M, N) block in every peer's staging area.
    const int64_t block_off = GATHER ? static_cast<int64_t>(p.M) * p.gx.cols[p.gx.rank] : 0;
    const uint32_t tempty_leader0 = map_to_cta(smem_u32(&tempty[0]), 0);
    int it = 0;
    for (int tile = pair; tile < p.num_tiles; tile += num_pairs, ++it) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      bool ok = mbar_wait(&tfull[buf], acc_phase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) {
          *abort_flag = 1;
          record_error(&g_error_word, (kSiteEpilogue << 8) | kErrReasonTimeout);
        }
        break;
      }
      tc_fence_after();
      const int64_t row_base =
          static_cast<int64_t>(tm) * 2 * BM + static_cast<int64_t>(rank) * BM + quarter * 32;
      const int64_t row = row_base + lane;
      const bool row_ok = row < p.M;
      T* orow = out + row * p.ldo;
      uint8_t* stg = epi_stage + (warp - 2) * EPI_STAGE_BYTES;
#pragma unroll 1
      for (int h = 0; h < BN; h += EPI_COLS) {
        const int hcol = tn * BN + h;  // first (local) column of this half tile
        // Full 128-column halves go through the staging buffer; ragged edges and
        // unaligned outputs take the per-thread path.
        const bool staged = vec_ok && hcol + EPI_COLS <= p.N;
        if constexpr (GATHER) {
          // the TMA stores of the previous block have read the buffer
          if (staged && p.tma_store) {
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
          }
        }
#pragma unroll 1
        for (int c = 0; c < EPI_COLS; c += 32) {
          uint32_t r[32];
          __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
          tmem_ld_32x32b_x32(
              tmem_base + buf * BN + h + c + (static_cast<uint32_t>(quarter * 32) << 16), r);
          tmem_ld_wait();
          const int col0 = hcol + c;
          if (staged) {
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float b0 = p.has_bias ? to_f32(bias[col0 + j]) : 0.f;
              const float b1 = p.has_bias ? to_f32(bias[col0 + j + 1]) : 0.f;
              const T lo = gemm_epilogue<T>(__uint_as_float(r[j]), p.has_bias, p.alpha, p.beta, b0);
              const T hi =
                  gemm_epilogue<T>(__uint_as_float(r[j + 1]), p.has_bias, p.alpha, p.beta, b1);
              packed[j / 2] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&lo)) |
                              (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
            }
            // Row `lane` of the stage, 16-byte chunk u stored at u ^ (lane & 15).
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int u = (c >> 3) + q;
              *reinterpret_cast<uint4*>(stg + stage_off<GATHER>(lane, u)) =
                  make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2],
                             packed[4 * q + 3]);
            }
            continue;
          }
          if (!row_ok || col0 >= p.N) continue;
          if (vec_ok && col0 + 32 <= p.N) {
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float b0 = p.has_bias ? to_f32(bias[col0 + j]) : 0.f;
              const float b1 = p.has_bias ? to_f32(bias[col0 + j + 1]) : 0.f;
              const T lo = gemm_epilogue<T>(__uint_as_float(r[j]), p.has_bias, p.alpha, p.beta, b0);
              const T hi =
                  gemm_epilogue<T>(__uint_as_float(r[j + 1]), p.has_bias, p.alpha, p.beta, b1);
              packed[j / 2] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&lo)) |
                              (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
            }
            uint4* dst = reinterpret_cast<uint4*>(orow + col0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2],
                                  packed[4 * q + 3]);
            }
            if constexpr (GATHER) {
              const int64_t off = block_off + row * p.N + col0;
              for (int j = 1; j < p.gx.world; ++j) {
                int rr = p.gx.rank + j;
                if (rr >= p.gx.world) rr -= p.gx.world;
                uint4* pd = reinterpret_cast<uint4*>(static_cast<T*>(p.gx.stages[rr]) + off);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  pd[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2],
                                     packed[4 * q + 3]);
                }
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (col0 + j < p.N) {
                const float bj = p.has_bias ? to_f32(bias[col0 + j]) : 0.f;
                const T v =
                    gemm_epilogue<T>(__uint_as_float(r[j]), p.has_bias, p.alpha, p.beta, bj);
                orow[col0 + j] = v;
                if constexpr (GATHER) {
                  const int64_t off = block_off + row * p.N + col0 + j;
                  for (int q = 1; q < p.gx.world; ++q) {
                    int rr = p.gx.rank + q;
                    if (rr >= p.gx.world) rr -= p.gx.world;
                    static_cast<T*>(p.gx.stages[rr])[off] = v;
                  }
                }
              }
            }
          }
        }
        if constexpr (GATHER) {
          if (staged && p.tma_store) {
            // The staged 32 x 128 block to every rank's copy, own output first: two
            // 64 x 32 boxes per destination, rows past M clipped by the copy engine.
            fence_proxy_async_smem();  // the lanes' shared-memory writes, to the async proxy
            __syncwarp();
            if (lane == 0 && row_base < p.M) {
              const int y = static_cast<int>(row_base);
              for (int j = 0; j < p.gx.world; ++j) {
                int d = p.gx.rank + j;
                if (d >= p.gx.world) d -= p.gx.world;
                tma_store_2d(&smap.m[d], stg, hcol, y);
                tma_store_2d(&smap.m[d], stg + 4096, hcol + 64, y);
              }
              bulk_commit_group();
            }
            __syncwarp();
            continue;
          }
        }
        if (staged) {
          // Write the staged 32 x 128 block: two rows per instruction, 16 threads x 16 B
          // = 256 contiguous bytes per row (and per row of each peer's staging block when
          // gathering).
          __syncwarp();
          const int half_row = lane >> 4;
          const int u = lane & 15;
#pragma unroll 4
          for (int rr = 0; rr < 32; rr += 2) {
            const int lr = rr + half_row;
            const int64_t grow = row_base + lr;
            const uint4 v =
                *reinterpret_cast<const uint4*>(stg + stage_off<GATHER>(lr, u));
            if (grow < p.M) {
              *reinterpret_cast<uint4*>(out + grow * p.ldo + hcol + u * 8) = v;
              if constexpr (GATHER) {
                const int64_t off = block_off + grow * p.N + hcol + u * 8;
                for (int j = 1; j < p.gx.world; ++j) {
                  int dr = p.gx.rank + j;
                  if (dr >= p.gx.world) dr -= p.gx.world;
                  *reinterpret_cast<uint4*>(static_cast<T*>(p.gx.stages[dr]) + off) = v;
                }
              }
            }
          }
          __syncwarp();  // the stage is rewritten by the next half
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + buf * 8);  // release on the leader
    }
    if constexpr (GATHER) {
      if (p.tma_store && lane == 0) {
        bulk_wait_all();             // this thread's TMA stores have written everything
        fence_proxy_async_global();  // ... ordered before its generic-proxy fence below
      }
      __syncwarp();
      __threadfence_system();  // this thread's peer stores, before the flag
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // the leader's MMAs are done and both epilogues have finished
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  if constexpr (GATHER) {
    if (threadIdx.x == 0) {
      // Every CTA's stores are fenced; the last CTA to count itself in publishes the
      // epoch to every rank and waits for every rank's.
      uint32_t* counter = p.gx.local + kFlagCounter;
      __threadfence_system();
      if (atomicAdd(counter, 1u) == gridDim.x - 1) {
        *counter = 0;  // the next call's CTAs start from zero (stream order)
        __threadfence_system();
        const uint32_t epoch = call_epoch(p.gx);
        for (int r = 0; r < p.gx.world; ++r) {
          st_release_sys(p.gx.flags[r] + kFlagExit + p.gx.rank, epoch);
        }
        for (int r = 0; r < p.gx.world; ++r) {
          if (!wait_flag_at_least(p.gx.flags[p.gx.rank] + kFlagExit + r, epoch)) {
            record_error(&g_error_word, (kSitePeerExit << 8) | kErrReasonTimeout);
            break;
          }
        }
      }
    }
  }
}

// Copies the blocks the other ranks stored into this rank's staging area into its
// output: source s's dense (M, cols[s+1] - cols[s]) block at element offset M * cols[s]
// becomes columns [cols[s], cols[s+1]) of `out` (row stride ldo).  16-byte vectors,
// UNPACK_UNROLL loads in flight per thread; blockIdx.y picks the source (every rank
// but this one).  The staging reads are single use (evict-first).
constexpr int UNPACK_THREADS = 256;
constexpr int UNPACK_UNROLL = 4;

__device__ __forceinline__ int64_t div_small(int64_t i, int64_t d) {
  // 32-bit division whenever both fit (d always does: it is a column count / 8)
  return (i >> 32) == 0 ? static_cast<int64_t>(static_cast<uint32_t>(i) / static_cast<uint32_t>(d))
                        : i / d;
}

__global__ void __launch_bounds__(UNPACK_THREADS)
    gather_unpack_kernel(const GatherArgs x, uint16_t* out, int64_t ldo, int64_t M) {
  int s = x.rank + 1 + static_cast<int>(blockIdx.y);
  if (s >= x.world) s -= x.world;
  const int64_t c0 = x.cols[s];
  const int64_t vpr = (x.cols[s + 1] - c0) >> 3;  // 16-byte vectors per row
  const int64_t total = M * vpr;
  const uint4* src =
      reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x.stages[x.rank]) + M * c0);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * UNPACK_THREADS;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * UNPACK_THREADS + threadIdx.x;
       base < total; base += UNPACK_UNROLL * stride) {
    uint4 v[UNPACK_UNROLL];
#pragma unroll
    for (int u = 0; u < UNPACK_UNROLL; ++u) {
      const int64_t i = base + u * stride;
      if (i < total) v[u] = __ldcs(src + i);
    }
#pragma unroll
    for (int u = 0; u < UNPACK_UNROLL; ++u) {
      const int64_t i = base + u * stride;
      if (i < total) {
        const int64_t r = div_small(i, vpr);
        *reinterpret_cast<uint4*>(out + r * ldo + c0 + (i - r * vpr) * 8) = v[u];
      }
    }
  }
}

// Stream-ordered barrier over the ranks of a GatherArgs (one warp): post the epoch to
// every rank's flag `slot` (entry or exit), then wait (bounded) for every rank's.
// With x.epoch == 0 the entry barrier takes the block's call count + 1 as the epoch
// and stores it back afterwards, so the call's later kernels (call_epoch) and the
// next call see it; ranks that make the same calls keep equal counts.
__global__ void peer_barrier_kernel(const GatherArgs x, int slot) {
  const int t = threadIdx.x;
  uint32_t* own = x.flags[x.rank];
  uint32_t epoch = x.epoch;
  if (epoch == 0) {
    epoch = *reinterpret_cast<volatile uint32_t*>(x.local + kFlagEpoch);
    if (slot == kFlagEntry) epoch += 1;
  }
  __threadfence_system();
  if (t < x.world) st_release_sys(x.flags[t] + slot + x.rank, epoch);
  __syncwarp();
  bool ok = true;
  if (t < x.world) ok = wait_flag_at_least(own + slot + t, epoch);
  if (!ok) {
    record_error(&g_error_word,
                 ((slot == kFlagEntry ? kSitePeerEntry : kSitePeerExit) << 8) | kErrReasonTimeout);
  }
  __syncwarp();
  if (x.epoch == 0 && slot == kFlagEntry && t == 0) x.local[kFlagEpoch] = epoch;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      return reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

}  // namespace tc

int encode_tiled16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides, const uint32_t* box, int dtype) {
  tc::EncodeTiledFn enc = tc::get_encode_fn();
  if (!enc) return set_error(BI_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const CUtensorMapDataType dt =
      dtype == BI_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    estr[i] = 1;
    if (i > 0) st[i - 1] = strides[i - 1];
  }
  CUresult r = enc(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st, bx,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return set_error(BI_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d), rank %d",
                     static_cast<int>(r), rank);
  }
  return BI_OK;
}

namespace tc {

// 2-D tensor map over a row-major (rows, cols) matrix of 16-bit elements with the
// given row stride (elements), box (box_cols x box_rows), 128-byte swizzle, and
// zero fill outside the matrix.
static int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                    int64_t row_stride, uint32_t box_cols, uint32_t box_rows, int dtype) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(BI_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const CUtensorMapDataType dt =
      dtype == BI_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return set_error(BI_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld",
                     static_cast<int>(r), static_cast<long long>(rows),
                     static_cast<long long>(cols));
  }
  return BI_OK;
}

// GATHER: the maps of the epilogue's TMA stores (see StoreMaps).  False, with nothing
// reported, when a destination does not meet the copy engine's rules (16-byte aligned
// base, row pitch a multiple of 16 bytes) -- the epilogue then stores with plain
// instructions, which write the same bytes.
static bool make_store_maps(StoreMaps* sm, const GemmArgs& g, const GatherArgs& x) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc || g.M <= 0 || g.N <= 0 || g.N % 8 != 0 || g.ldo % 8 != 0) return false;
  const int64_t block_off = g.M * x.cols[x.rank];  // elements
  for (int d = 0; d < x.world; ++d) {
    void* base = d == x.rank ? g.out
                             : static_cast<void*>(static_cast<uint16_t*>(x.stages[d]) + block_off);
    const int64_t pitch = d == x.rank ? g.ldo : g.N;
    if (base == nullptr || (reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(g.N), static_cast<cuuint64_t>(g.M)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch) * 2};
    cuuint32_t box[2] = {64, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&sm->m[d], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base, dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
  }
  return true;
}

// Raster of the persistent schedule: consecutive tile indices walk group_m pair-tiles
// down M for one column tile before moving along N, so the pairs running at once share
// a few W column slices in L2.  It decides which pair computes a tile, never a bit.
// Group 8 (16 from 32 row tiles up: measured +2.7 % at M = 16384 on (8192, 57344)).
static int group_m_for(int tiles_m) {
  if (tiles_m >= 32) return 16;
  return tiles_m < 8 ? tiles_m : 8;
}

template <typename T, bool B_NK, bool GATHER, typename R>
static int launch_ring(const GemmArgs& g, const GatherArgs* gx, cudaStream_t stream) {
  CUtensorMap ma, mb;
  int st = make_map(&ma, g.a, g.M, g.K, g.lda, BK, R::A_ROWS, g.dtype);
  if (st) return st;
  if (B_NK) {
    st = make_map(&mb, g.b, g.N, g.K, g.ldb, BK, R::BN_CTA, g.dtype);
  } else {
    st = make_map(&mb, g.b, g.K, g.N, g.ldb, 64, BK, g.dtype);
  }
  if (st) return st;

  auto kern = gemm_tc_kernel<T, B_NK, GATHER, R>;
  // The attribute is per device; setting it again is cheap and capture-safe.
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       R::SMEM_BYTES);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm_tc)");

  Params p;
  p.bias = g.bias;
  p.out = g.out;
  p.ldo = g.ldo;
  p.M = static_cast<int>(g.M);
  p.N = static_cast<int>(g.N);
  p.K = static_cast<int>(g.K);
  p.alpha = g.alpha;
  p.beta = g.beta;
  p.has_bias = g.bias != nullptr;
  p.tiles_m = static_cast<int>((g.M + 2 * BM - 1) / (2 * BM));
  p.tiles_n = static_cast<int>((g.N + R::BN - 1) / R::BN);
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.group_m = group_m_for(p.tiles_m);
  StoreMaps sm;
  memset(&sm, 0, sizeof(sm));
  p.tma_store = 0;
  if (gx != nullptr) {
    p.gx = *gx;
    if (GATHER) p.tma_store = make_store_maps(&sm, g, *gx) ? 1 : 0;
  } else {
    p.gx = GatherArgs{};
  }
  const int max_pairs = device_sm_count() / 2;
  const int pairs = p.num_tiles < max_pairs ? p.num_tiles : max_pairs;
  kern<<<2 * pairs, NUM_THREADS, R::SMEM_BYTES, stream>>>(ma, mb, p, sm);
  return cuda_status(cudaGetLastError(), "gemm_tc launch");
}

// The ring is the only thing M selects: a thin one when every row of the problem fits
// in the 16-row A box (decode), else the wide one.  Both run the same UMMAs.
template <typename T, bool B_NK, bool GATHER>
static int launch_typed(const GemmArgs& g, const GatherArgs* gx, cudaStream_t stream) {
  return g.M <= THIN_MAX_M ? launch_ring<T, B_NK, GATHER, ThinRing>(g, gx, stream)
                           : launch_ring<T, B_NK, GATHER, WideRing>(g, gx, stream);
}

template <bool GATHER>
static int dispatch(const GemmArgs& g, const GatherArgs* gx, cudaStream_t stream) {
  if (g.dtype == BI_BF16) {
    return g.b_is_nk ? launch_typed<__nv_bfloat16, true, GATHER>(g, gx, stream)
                     : launch_typed<__nv_bfloat16, false, GATHER>(g, gx, stream);
  }
  if (g.dtype == BI_F16) {
    return g.b_is_nk ? launch_typed<__half, true, GATHER>(g, gx, stream)
                     : launch_typed<__half, false, GATHER>(g, gx, stream);
  }
  return set_error(BI_ERR_UNSUPPORTED, "tensor-core route takes fp16 or bf16");
}

}  // namespace tc

int launch_gemm_tc(const GemmArgs& g, cudaStream_t stream) {
  if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX) {
    return set_error(BI_ERR_UNSUPPORTED, "dimensions above 2^31 are not supported");
  }
  return tc::dispatch<false>(g, nullptr, stream);
}

int launch_gemm_tc_allgather(const GemmArgs& g, const GatherArgs& x, void* out_base,
                             cudaStream_t stream, bool unpack) {
  if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX) {
    return set_error(BI_ERR_UNSUPPORTED, "dimensions above 2^31 are not supported");
  }
  int st;
  if (g.M == 0 || g.N == 0) {
    // An empty shard computes nothing but still posts and awaits the exit epoch the
    // peers' GEMMs wait for.
    tc::peer_barrier_kernel<<<1, 32, 0, stream>>>(x, kFlagExit);
    st = cuda_status(cudaGetLastError(), "peer exit launch");
  } else {
    st = tc::dispatch<true>(g, &x, stream);
  }
  if (st || !unpack) return st;
  // Every peer has posted its exit epoch once the kernel above ends: unpack their blocks.
  return launch_gather_unpack(x, out_base, g.ldo, g.M, stream);
}

int launch_gather_unpack(const GatherArgs& x, void* out_base, int64_t ldo, int64_t M,
                         cudaStream_t stream) {
  if (M == 0 || x.world == 1) return BI_OK;
  int64_t most = 0;
  for (int r = 0; r < x.world; ++r) {
    if (r != x.rank) most = std::max(most, M * ((x.cols[r + 1] - x.cols[r]) >> 3));
  }
  if (most == 0) return BI_OK;
  const int64_t per_cta = static_cast<int64_t>(tc::UNPACK_THREADS) * tc::UNPACK_UNROLL;
  const int64_t want = (most + per_cta - 1) / per_cta;
  const int ctas = static_cast<int>(std::min<int64_t>(want, 4 * device_sm_count()));
  tc::gather_unpack_kernel<<<dim3(ctas, x.world - 1), tc::UNPACK_THREADS, 0, stream>>>(
      x, static_cast<uint16_t*>(out_base), ldo, M);
  return cuda_status(cudaGetLastError(), "gather unpack launch");
}

int launch_peer_barrier(const GatherArgs& x, cudaStream_t stream) {
  tc::peer_barrier_kernel<<<1, 32, 0, stream>>>(x, kFlagEntry);
  return cuda_status(cudaGetLastError(), "peer barrier launch");
}

// Device address of `device`'s copy of g_static_flag_block.  Looked up once per device,
// with that device current (the host-side name of a __device__ array is only a
// stand-in for it), then cached.
int static_flag_block(int device, void** out) {
  static std::mutex mu;
  static void* cache[64] = {};
  if (device < 0 || device >= 64) return set_error(BI_ERR_INVALID, "device %d out of range", device);
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == nullptr) {
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    if (cur != device) {
      e = cudaSetDevice(device);
      if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice(static flag block)");
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_flag_block);
    const cudaError_t back = cur != device ? cudaSetDevice(cur) : cudaSuccess;
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(static flag block)");
    if (back != cudaSuccess) return cuda_status(back, "cudaSetDevice(restore)");
    cache[device] = p;
  }
  *out = cache[device];
  return BI_OK;
}

unsigned read_error_gemm_tc(bool clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, tc::g_error_word, sizeof(v));
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(tc::g_error_word, &z, sizeof(z));
  }
  return v;
}

}  // namespace bi
