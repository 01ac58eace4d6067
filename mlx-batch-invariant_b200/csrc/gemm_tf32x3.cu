// Batch-invariant float32 GEMM on the tensor cores: three tf32 products per K step
// (tcgen05.mma kind::tf32, 2-SM, M=256, N=256, K=8) with fp32 accumulation in TMEM.
//
// Each fp32 operand x is split exactly into big + small: big keeps x's sign, exponent
// and top 10 mantissa bits (the low 13 bits cleared -- a tf32 value, so the tensor
// core takes it as is whatever its input conversion), small = x - big (exact in fp32,
// at most 2^-10 |x|).  Per K=8 step the pair accumulates, in this order,
//     a_big * b_big,  a_big * b_small,  a_small * b_big
// and drops a_small * b_small (about 2^-20 of a product).  The tensor core keeps the
// top 11 significant bits of small, so each product is within about 2^-19 of a * b.
// The tensor core's fp32 accumulator drifts by a fraction of an ulp on every MMA
// (measured: error growing linearly in K, 2.2e-4 normwise at K = 28672 when one
// accumulator takes all of K), so K is summed in chunks of 256 in TMEM and the
// epilogue adds the chunk sums in K order in fp32 with round to nearest, keeping the
// running sum in the output; the GPU tests hold it to 5e-6 normwise against float64.
//
// Invariance: as in gemm_tc_kernel -- one pair owns an output element's whole K
// reduction, the tile (256 x 256), K block (32) and instruction sequence are fixed,
// so an element's bits do not depend on M, on its row's position or on the other rows.
// There is one ring for every M (no decode-sized variant).
//
// Structure (clusters of two CTAs, persistent, one per SM):
//   warp 0      TMA producer: this CTA's 128 rows of A and 128 columns of B per
//               32-deep K block, completing on this CTA's own full barrier.
//   warp 1      TMEM allocator and, in the leader, the UMMA issuer (3 x 4 UMMAs per
//               K block, after both CTAs' converters have signalled the stage).
//   warps 2..5  epilogue: tcgen05.ld of each 256-deep K chunk, added to the running
//               sum in the output; after the last, alpha / beta / bias in fp32.
//   warps 6..9  converters: rewrite the stage's A and B in place as big and write
//               small beside them, fence to the async proxy, arrive on the leader.
// Every mbarrier wait is bounded; a wait that gives up records the device error word.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace bi {
namespace tf3 {

constexpr int BM = 128;          // rows per CTA (the pair covers 2*BM)
constexpr int BN = 256;          // columns per pair tile
constexpr int BN_CTA = BN / 2;   // B columns each CTA loads
constexpr int BK = 32;           // 32 fp32 = one 128-byte swizzle row
constexpr int UMMA_K = 8;        // kind::tf32: 8 elements (32 bytes) per step
constexpr int STAGES = 3;
constexpr int ACC_BUFS = 2;
// K blocks summed in one TMEM accumulator before the epilogue adds the chunk into the
// running fp32 sum (round to nearest): the tensor core's fp32 accumulation drifts by a
// fraction of an ulp per MMA, so its error grows with the MMAs per chunk, not with K.
constexpr int KB_PER_CHUNK = 8;  // 256 of K
constexpr int TMEM_COLS = ACC_BUFS * BN;  // 512
constexpr int OP_BYTES = BM * BK * 4;     // 16 KiB: one operand tile of one CTA
constexpr int STAGE_BYTES = 4 * OP_BYTES; // A, B (rewritten as big), A small, B small
constexpr int EPI_WARPS = 4;
constexpr int CONV_WARPS = 4;
constexpr int NUM_THREADS = 32 * (2 + EPI_WARPS + CONV_WARPS);  // 320
constexpr int EPI_COLS = 32;                                   // fp32 columns per staged block
constexpr int EPI_STAGE_BYTES = 32 * EPI_COLS * 4;             // 4 KiB per epilogue warp
constexpr int NUM_BARRIERS = 3 * STAGES + 2 * ACC_BUFS + 1;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_WARPS * EPI_STAGE_BYTES +
                           NUM_BARRIERS * 8 + 16;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory above the per-CTA limit");
constexpr uint16_t PAIR_MASK = 0x3;

enum : unsigned {
  kSiteProducer = 1,
  kSiteMma = 2,
  kSiteEpilogue = 3,
  kSiteDrain = 4,
  kSiteConvert = 5
};

__device__ unsigned g_error_word = 0;

struct Params {
  const float* bias;
  float* out;
  int64_t ldo;
  int M, N, K;
  float alpha, beta;
  int has_bias;
  int tiles_m, tiles_n, num_tiles, group_m;
};

__device__ __forceinline__ void tile_coords(int tile, const Params& p, int& tm, int& tn) {
  const int per_group = p.group_m * p.tiles_n;
  const int group = tile / per_group;
  const int first_m = group * p.group_m;
  const int rows = min(p.tiles_m - first_m, p.group_m);
  const int in_group = tile - group * per_group;
  tm = first_m + in_group % rows;
  tn = in_group / rows;
}

// 2-SM UMMA, kind::tf32 (32-bit operands in shared memory, fp32 accumulation).
__device__ __forceinline__ void umma_tf32_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::tf32: A and B tf32 (format 2), D fp32.
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t b_mn_major, uint32_t m, uint32_t n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (b_mn_major << 16) | ((n >> 3) << 17) |
         ((m >> 4) << 24);
}

// Waits with cluster-scope acquire: the arrivals may come from the peer CTA, whose
// shared-memory writes the leader's UMMAs then read.
__device__ __forceinline__ bool mbar_try_wait_acq_cluster(uint32_t bar_addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait_acq_cluster(uint64_t* bar, uint32_t parity,
                                                      const volatile int* abort_flag) {
  const uint32_t addr = smem_u32(bar);
  const long long start = clock64();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait_acq_cluster(addr, parity)) return true;
    if ((it & 63u) == 63u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (clock64() - start > kWaitBudgetCycles) return false;
    }
  }
}

// x -> (big, small): big = x with its low 13 mantissa bits cleared, small = x - big.
__device__ __forceinline__ void split4(const uint4 x, uint4& big, uint4& small) {
  const uint32_t m = 0xffffe000u;
  big = make_uint4(x.x & m, x.y & m, x.z & m, x.w & m);
  small = make_uint4(__float_as_uint(__fsub_rn(__uint_as_float(x.x), __uint_as_float(big.x))),
                     __float_as_uint(__fsub_rn(__uint_as_float(x.y), __uint_as_float(big.y))),
                     __float_as_uint(__fsub_rn(__uint_as_float(x.z), __uint_as_float(big.z))),
                     __float_as_uint(__fsub_rn(__uint_as_float(x.w), __uint_as_float(big.w))));
}

template <bool B_NK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_b, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // stage s: [A (big after conversion) | B (big) | A small | B small], 16 KiB each
  uint8_t* epi_stage = smem + STAGES * STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + EPI_WARPS * EPI_STAGE_BYTES);
  uint64_t* full = bars;                          // this CTA's TMA bytes landed
  uint64_t* conv = bars + STAGES;                 // leader: both CTAs converted (8 arrivals)
  uint64_t* empty = bars + 2 * STAGES;            // MMAs done with the stage (both CTAs)
  uint64_t* tfull = bars + 3 * STAGES;            // accumulator ready (both CTAs)
  uint64_t* tempty = bars + 3 * STAGES + ACC_BUFS;  // accumulator drained (leader)
  uint64_t* mma_done = bars + 3 * STAGES + 2 * ACC_BUFS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARRIERS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 2 * CONV_WARPS);
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
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (p.K + BK - 1) / BK;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs, each into its own stages) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs) {
        int tm, tn;
        tile_coords(tile, p, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint64_t* bar = &full[stage];
          mbar_arrive_expect_tx(bar, 2 * OP_BYTES);
          uint8_t* st = smem + stage * STAGE_BYTES;
          tma_load_2d(st, &tmap_a, bar, kb * BK, tm * 2 * BM + static_cast<int>(rank) * BM);
          const int n0 = tn * BN + static_cast<int>(rank) * BN_CTA;
          if (B_NK) {
            tma_load_2d(st + OP_BYTES, &tmap_b, bar, kb * BK, n0);
          } else {
            // (K, N) row-major B: four 32-column slabs, each 32 k-rows of 128 bytes
#pragma unroll
            for (int j = 0; j < BN_CTA / 32; ++j) {
              tma_load_2d(st + OP_BYTES + j * (32 * BK * 4), &tmap_b, bar, n0 + j * 32, kb * BK);
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
        if (issued_any) sleep_ns(200000);
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer (leader only) ----------------
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(B_NK ? 0u : 1u, 2 * BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;  // chunks issued (each fills one accumulator buffer)
      for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs) {
       for (int kc = 0; kc < num_kb && ok; kc += KB_PER_CHUNK, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[buf], acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        const int kc_end = min(kc + KB_PER_CHUNK, num_kb);
        for (int kb = kc; kb < kc_end; ++kb) {
          if (!mbar_wait_acq_cluster(&conv[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t a_big = st, b_big = st + OP_BYTES;
          const uint32_t a_small = st + 2 * OP_BYTES, b_small = st + 3 * OP_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // K-major, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart; the
            // K=8 step moves 32 bytes along the row.  MN-major B (32-bit operands take
            // only the 128-byte swizzle with 32-byte atoms, layout type 1): 32-column
            // slabs 4 KiB apart (LBO), 4-k-row groups 512 B apart (SBO); the K=8 step
            // moves 8 k-rows, 1024 B.
            const uint32_t ko = k * UMMA_K * 4;
            const uint64_t ab = umma_smem_desc(a_big + ko, 16, 1024, 2);
            const uint64_t as = umma_smem_desc(a_small + ko, 16, 1024, 2);
            uint64_t bb, bs;
            if (B_NK) {
              bb = umma_smem_desc(b_big + ko, 16, 1024, 2);
              bs = umma_smem_desc(b_small + ko, 16, 1024, 2);
            } else {
              bb = umma_smem_desc(b_big + k * UMMA_K * 128, 32 * BK * 4, 512, 1);
              bs = umma_smem_desc(b_small + k * UMMA_K * 128, 32 * BK * 4, 512, 1);
            }
            umma_tf32_pair(d_tmem, ab, bb, idesc, ((kb - kc) | k) != 0 ? 1u : 0u);
            umma_tf32_pair(d_tmem, ab, bs, idesc, 1u);
            umma_tf32_pair(d_tmem, as, bb, idesc, 1u);
          }
          umma_commit_pair(&empty[stage], PAIR_MASK);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[buf], PAIR_MASK);
       }
      }
      if (!ok) {
        *abort_flag = 1;
        record_error(&g_error_word, (kSiteMma << 8) | kErrReasonTimeout);
      }
      umma_commit_pair(mma_done, 0x1);
      if (!mbar_wait(mma_done, 0, nullptr)) {
        record_error(&g_error_word, (kSiteDrain << 8) | kErrReasonTimeout);
      }
    }
  } else if (warp >= 2 + EPI_WARPS) {
    // ---------------- converters (warps 6..9, both CTAs) ----------------
    const int ct = threadIdx.x - 32 * (2 + EPI_WARPS);  // 0..127
    const uint32_t conv_leader0 = map_to_cta(smem_u32(&conv[0]), 0);
    int stage = 0;
    uint32_t phase = 0;
    const int total = p.num_tiles;
    for (int tile = pair; tile < total; tile += num_pairs) {
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        ok = mbar_wait(&full[stage], phase, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        uint4* raw = reinterpret_cast<uint4*>(smem + stage * STAGE_BYTES);  // A then B
        uint4* small = reinterpret_cast<uint4*>(smem + stage * STAGE_BYTES + 2 * OP_BYTES);
        // 2 * 16 KiB = 2048 16-byte chunks, 16 per thread, consecutive threads on
        // consecutive chunks (conflict-free); small sits at the same offset as its x,
        // so it inherits the swizzled layout the UMMA descriptors expect.
#pragma unroll 4
        for (int i = ct; i < 2 * OP_BYTES / 16; i += 32 * CONV_WARPS) {
          uint4 big, sm;
          split4(raw[i], big, sm);
          raw[i] = big;
          small[i] = sm;
        }
        fence_proxy_async_smem();  // the writes above, before the UMMAs read them
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(conv_leader0 + stage * 8);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {
        if (lane == 0) {
          *abort_flag = 1;
          record_error(&g_error_word, (kSiteConvert << 8) | kErrReasonTimeout);
        }
        break;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    const int quarter = warp & 3;
    float* out = p.out;
    const float* bias = p.bias;
    const bool vec_ok = (p.ldo % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
    const uint32_t tempty_leader0 = map_to_cta(smem_u32(&tempty[0]), 0);
    uint8_t* stg = epi_stage + (warp - 2) * EPI_STAGE_BYTES;
    int it = 0;  // chunks consumed
    bool ok = true;
    for (int tile = pair; tile < p.num_tiles && ok; tile += num_pairs) {
      int tm, tn;
      tile_coords(tile, p, tm, tn);
      const int64_t row_base =
          static_cast<int64_t>(tm) * 2 * BM + static_cast<int64_t>(rank) * BM + quarter * 32;
      const int64_t row = row_base + lane;
      for (int kc = 0; kc < num_kb; kc += KB_PER_CHUNK, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        ok = mbar_wait(&tfull[buf], acc_phase, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
          if (lane == 0) {
            *abort_flag = 1;
            record_error(&g_error_word, (kSiteEpilogue << 8) | kErrReasonTimeout);
          }
          break;
        }
        tc_fence_after();
        // Chunk sums enter the output in K order: the first is stored as is, each later
        // one is added (fp32, round to nearest) to the running sum the same thread
        // stored before, and the last one's total takes alpha / beta / bias and the
        // final store.  The thread that owns an element is the same in every chunk.
        const bool first = kc == 0;
        const bool last = kc + KB_PER_CHUNK >= num_kb;
#pragma unroll 1
        for (int c = 0; c < BN; c += EPI_COLS) {
          const int col0 = tn * BN + c;
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tmem_base + buf * BN + c + (static_cast<uint32_t>(quarter * 32) << 16),
                             r);
          tmem_ld_wait();
          if (col0 >= p.N) continue;
          if (vec_ok && col0 + 32 <= p.N) {
            // stage the warp's 32 x 32 chunk block (row `lane`, 16-byte piece u at
            // u ^ (lane & 7)); then lane (lr, u) handles 4 columns of row lr, 4 rows at a
            // time, 128 contiguous bytes per row
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              *reinterpret_cast<uint4*>(stg + lane * 128 + ((u ^ (lane & 7)) << 4)) =
                  make_uint4(r[4 * u], r[4 * u + 1], r[4 * u + 2], r[4 * u + 3]);
            }
            __syncwarp();
            const int u = lane & 7;
            const int cc = col0 + u * 4;
            float4 prev[8];
            if (!first) {
#pragma unroll
              for (int rr = 0; rr < 8; ++rr) {
                const int64_t grow = row_base + rr * 4 + (lane >> 3);
                prev[rr] = grow < p.M ? *reinterpret_cast<const float4*>(out + grow * p.ldo + cc)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
#pragma unroll
            for (int rr = 0; rr < 8; ++rr) {
              const int lr = rr * 4 + (lane >> 3);
              const int64_t grow = row_base + lr;
              float4 val =
                  *reinterpret_cast<const float4*>(stg + lr * 128 + ((u ^ (lr & 7)) << 4));
              if (!first) {
                val.x = __fadd_rn(prev[rr].x, val.x);
                val.y = __fadd_rn(prev[rr].y, val.y);
                val.z = __fadd_rn(prev[rr].z, val.z);
                val.w = __fadd_rn(prev[rr].w, val.w);
              }
              if (last) {
                const float b0 = p.has_bias ? bias[cc] : 0.f;
                const float b1 = p.has_bias ? bias[cc + 1] : 0.f;
                const float b2 = p.has_bias ? bias[cc + 2] : 0.f;
                const float b3 = p.has_bias ? bias[cc + 3] : 0.f;
                val.x = gemm_epilogue<float>(val.x, p.has_bias, p.alpha, p.beta, b0);
                val.y = gemm_epilogue<float>(val.y, p.has_bias, p.alpha, p.beta, b1);
                val.z = gemm_epilogue<float>(val.z, p.has_bias, p.alpha, p.beta, b2);
                val.w = gemm_epilogue<float>(val.w, p.has_bias, p.alpha, p.beta, b3);
              }
              if (grow < p.M) *reinterpret_cast<float4*>(out + grow * p.ldo + cc) = val;
            }
            __syncwarp();
          } else if (row < p.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (col0 + j < p.N) {
                float v = __uint_as_float(r[j]);
                if (!first) v = __fadd_rn(out[row * p.ldo + col0 + j], v);
                if (last) {
                  v = gemm_epilogue<float>(v, p.has_bias, p.alpha, p.beta,
                                           p.has_bias ? bias[col0 + j] : 0.f);
                }
                out[row * p.ldo + col0 + j] = v;
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader0 + buf * 8);
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

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

// 2-D tensor map over a row-major (rows, cols) fp32 matrix, box (box_cols x box_rows),
// 128-byte swizzle, zero fill outside the matrix.
static int make_map_f32(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                        int64_t row_stride, uint32_t box_cols, uint32_t box_rows,
                        CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(BI_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return set_error(BI_ERR_INVALID, "cuTensorMapEncodeTiled (fp32) failed (%d) rows=%lld cols=%lld",
                     static_cast<int>(r), static_cast<long long>(rows),
                     static_cast<long long>(cols));
  }
  return BI_OK;
}

template <bool B_NK>
static int launch(const GemmArgs& g, cudaStream_t stream) {
  CUtensorMap ma, mb;
  int st = make_map_f32(&ma, g.a, g.M, g.K, g.lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  // a (K, N) B is MN-major in shared memory: 128-byte swizzle with 32-byte atoms
  st = B_NK ? make_map_f32(&mb, g.b, g.N, g.K, g.ldb, BK, BN_CTA, CU_TENSOR_MAP_SWIZZLE_128B)
            : make_map_f32(&mb, g.b, g.K, g.N, g.ldb, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  if (st) return st;
  auto kern = gemm_tf32x3_kernel<B_NK>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_BYTES);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm_tf32x3)");
  Params p;
  p.bias = static_cast<const float*>(g.bias);
  p.out = static_cast<float*>(g.out);
  p.ldo = g.ldo;
  p.M = static_cast<int>(g.M);
  p.N = static_cast<int>(g.N);
  p.K = static_cast<int>(g.K);
  p.alpha = g.alpha;
  p.beta = g.beta;
  p.has_bias = g.bias != nullptr;
  p.tiles_m = static_cast<int>((g.M + 2 * BM - 1) / (2 * BM));
  p.tiles_n = static_cast<int>((g.N + BN - 1) / BN);
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.group_m = p.tiles_m >= 32 ? 16 : std::min(p.tiles_m, 8);
  const int max_pairs = device_sm_count() / 2;
  const int pairs = p.num_tiles < max_pairs ? p.num_tiles : max_pairs;
  kern<<<2 * pairs, NUM_THREADS, SMEM_BYTES, stream>>>(ma, mb, p);
  return cuda_status(cudaGetLastError(), "gemm_tf32x3 launch");
}

}  // namespace tf3

int launch_gemm_tf32x3(const GemmArgs& g, cudaStream_t stream) {
  if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX) {
    return set_error(BI_ERR_UNSUPPORTED, "dimensions above 2^31 are not supported");
  }
  return g.b_is_nk ? tf3::launch<true>(g, stream) : tf3::launch<false>(g, stream);
}

unsigned read_error_tf32x3(bool clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, tf3::g_error_word, sizeof(v));
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(tf3::g_error_word, &z, sizeof(z));
  }
  return v;
}

}  // namespace bi
