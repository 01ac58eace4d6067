// Batch-invariant GEMM on the CUDA cores: the route for fp32 inputs, and for fp16 /
// bf16 shapes the tensor-core route cannot take (K or the B row stride not a
// multiple of 8 elements, K = 0).
//
// Order of the reduction, per output element (the reference's k0 / kk structure of
// 8-deep MMA steps, mlx_batch_invariant/_gemm.py:62-104): K is cut into slices of 8,
// k ascending; each slice is summed in order into a fresh fp32 partial with fmaf
// (p = fmaf(a[k], b[k], p)), and the partial is added to the fp32 accumulator
// (acc = acc + p).  This is exactly the host oracle's order, so the route is bit-exact
// against it.  Each output element is one thread's sequence of scalar operations, so
// the thread layout cannot change a bit: a 128 x 128 x 8 CTA tile in general, and for
// up to 64 rows with (N, K) weights a warp per output column (gemm_simt_rows_kernel).
// Each element's K reduction stays in one thread; nothing in the arithmetic depends
// on M.
#include "common.cuh"
#include "internal.h"

namespace bi {
namespace simt {

constexpr int BM = kSimtBM;
constexpr int BN = kSimtBN;
constexpr int BK = kSimtBK;
constexpr int NUM_THREADS = 256;

struct Params {
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  const void* bias;
  void* out;
  int64_t ldo;
  int M, N, K;
  float alpha, beta;
  int has_bias;
};

template <typename T, bool B_NK>
__device__ __forceinline__ void load_tile(const Params& p, int row0, int col0, int k0, int tid,
                                          float (&ra)[4], float (&rb)[4]) {
  const T* A = static_cast<const T*>(p.a);
  const T* B = static_cast<const T*>(p.b);
  // A: row tid/2, k k0 + (tid%2)*4 .. +3
  {
    const int r = row0 + (tid >> 1);
    const int kc = k0 + (tid & 1) * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int k = kc + q;
      ra[q] = (r < p.M && k < p.K) ? to_f32(A[static_cast<int64_t>(r) * p.lda + k]) : 0.f;
    }
  }
  if (B_NK) {
    const int n = col0 + (tid >> 1);
    const int kc = k0 + (tid & 1) * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int k = kc + q;
      rb[q] = (n < p.N && k < p.K) ? to_f32(B[static_cast<int64_t>(n) * p.ldb + k]) : 0.f;
    }
  } else {
    const int k = k0 + (tid >> 5);
    const int nc = col0 + (tid & 31) * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int n = nc + q;
      rb[q] = (n < p.N && k < p.K) ? to_f32(B[static_cast<int64_t>(k) * p.ldb + n]) : 0.f;
    }
  }
}

template <bool B_NK>
__device__ __forceinline__ void store_tile(float (*As)[BM], float (*Bs)[BN], int tid,
                                           const float (&ra)[4], const float (&rb)[4]) {
  {
    const int r = tid >> 1;
    const int kc = (tid & 1) * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) As[kc + q][r] = ra[q];
  }
  if (B_NK) {
    const int n = tid >> 1;
    const int kc = (tid & 1) * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) Bs[kc + q][n] = rb[q];
  } else {
    const int k = tid >> 5;
    const int nc = (tid & 31) * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) Bs[k][nc + q] = rb[q];
  }
}

template <typename T, bool B_NK>
__global__ void __launch_bounds__(NUM_THREADS) gemm_simt_kernel(const Params p) {
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid & 15;
  const int ty = tid >> 4;
  const int row0 = blockIdx.y * BM;
  const int col0 = blockIdx.x * BN;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int num_kb = (p.K + BK - 1) / BK;
  float ra[4], rb[4];
  if (num_kb > 0) {
    load_tile<T, B_NK>(p, row0, col0, 0, tid, ra, rb);
    store_tile<B_NK>(As[0], Bs[0], tid, ra, rb);
  }
  __syncthreads();

  for (int kb = 0; kb < num_kb; ++kb) {
    const int cur = kb & 1;
    if (kb + 1 < num_kb) load_tile<T, B_NK>(p, row0, col0, (kb + 1) * BK, tid, ra, rb);
    float part[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) part[i][j] = 0.f;
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) part[i][j] = __fmaf_rn(a[i], b[j], part[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = __fadd_rn(acc[i][j], part[i][j]);
    if (kb + 1 < num_kb) store_tile<B_NK>(As[cur ^ 1], Bs[cur ^ 1], tid, ra, rb);
    __syncthreads();
  }

  const T* bias = static_cast<const T*>(p.bias);
  T* out = static_cast<T*>(p.out);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = row0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (r >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = col0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (c >= p.N) continue;
      const float bj = p.has_bias ? to_f32(bias[c]) : 0.f;
      out[static_cast<int64_t>(r) * p.ldo + c] =
          gemm_epilogue<T>(acc[i][j], p.has_bias, p.alpha, p.beta, bj);
    }
  }
}

// ---------------------------------------------------------------------------
// Few rows (M <= ROWS_MAX_M = 64), (N, K) weights: one warp per output column.
//
// Same arithmetic per element as gemm_simt_kernel -- slice partials p_s =
// fmaf-chain over k = 8s..8s+7 (zero past K) from a fresh +0, then acc = acc + p_s in
// slice order -- laid out for streaming W: lane l computes the partials of slices
// 32c + l of every row from one coalesced 32-byte read of the column's weight row, the
// partials go through shared memory, and lane m adds row m's in order.  The tiled
// kernel above pads M to 128 rows per CTA; this one reads each weight once per column.
constexpr int ROWS_MAX_M = 64;
// Warps per CTA for a MAXM-row instantiation: the partials buffer stays 33 KB.
constexpr int rows_warps(int maxm) { return 256 / maxm; }

// Elements k0 .. k0+7 of a row as fp32, zero past K.  VEC: the 8 elements are one
// aligned 16- or 32-byte run whenever k0 + 8 <= K.
template <typename T, bool VEC>
__device__ __forceinline__ void load8(const T* row, int k0, int K, float (&v)[8]) {
  if (VEC && k0 + 8 <= K) {
    if constexpr (sizeof(T) == 4) {
      const float4 x = *reinterpret_cast<const float4*>(row + k0);
      const float4 y = *reinterpret_cast<const float4*>(row + k0 + 4);
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
      v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
    } else {
      const uint4 x = *reinterpret_cast<const uint4*>(row + k0);
      const T* h = reinterpret_cast<const T*>(&x);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = to_f32(h[j]);
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = (k0 + j < K) ? to_f32(row[k0 + j]) : 0.f;
}

// Chunks of 32 slices whose weights a lane keeps in flight ahead of the one it uses.
constexpr int ROWS_PREFETCH = 4;

// MAXM (32 or 64): the rows this instantiation holds; lane l folds rows l and l + 32.
template <typename T, bool VEC, int MAXM>
__global__ void __launch_bounds__(32 * rows_warps(MAXM)) gemm_simt_rows_kernel(const Params p) {
  constexpr int RB = MAXM / 32;  // rows folded per lane
  constexpr int ROWS_WARPS = rows_warps(MAXM);
  __shared__ float part_s[ROWS_WARPS][MAXM][33];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * ROWS_WARPS + warp;
  if (n >= p.N) return;  // whole warps only; no CTA-wide barrier follows
  const T* A = static_cast<const T*>(p.a);
  const T* Bn = static_cast<const T*>(p.b) + static_cast<int64_t>(n) * p.ldb;
  const int slices = (p.K + BK - 1) / BK;
  float (*ps)[33] = part_s[warp];
  float acc[RB];  // acc[r]: row lane + 32 r
#pragma unroll
  for (int r = 0; r < RB; ++r) acc[r] = 0.f;
  float w[ROWS_PREFETCH][8];  // slot u holds the weights of chunk (index mod PF) == u
#pragma unroll
  for (int u = 0; u < ROWS_PREFETCH; ++u) load8<T, VEC>(Bn, BK * (32 * u + lane), p.K, w[u]);
  for (int c0 = 0; c0 < slices; c0 += 32 * ROWS_PREFETCH) {
#pragma unroll
    for (int u = 0; u < ROWS_PREFETCH; ++u) {
      const int cc = c0 + 32 * u;  // first slice of this chunk (warp-uniform)
      if (cc < slices) {
        const int s = cc + lane;
        for (int m = 0; m < p.M; ++m) {
          float a[8];
          load8<T, VEC>(A + static_cast<int64_t>(m) * p.lda, BK * s, p.K, a);
          float part = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) part = __fmaf_rn(a[j], w[u][j], part);
          ps[m][lane] = part;
        }
        // refill the slot with the chunk PF ahead (zeros past K)
        load8<T, VEC>(Bn, BK * (s + 32 * ROWS_PREFETCH), p.K, w[u]);
        __syncwarp();
        const int cnt = slices - cc < 32 ? slices - cc : 32;
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          const int row = lane + 32 * r;
          if (row < p.M) {
            // all 32 loads first, then the adds strictly in slice order
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = ps[row][i];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (i < cnt) acc[r] = __fadd_rn(acc[r], v[i]);
            }
          }
        }
        __syncwarp();
      }
    }
  }
  const T* bias = static_cast<const T*>(p.bias);
  const float bj = p.has_bias ? to_f32(bias[n]) : 0.f;
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    const int row = lane + 32 * r;
    if (row < p.M) {
      static_cast<T*>(p.out)[static_cast<int64_t>(row) * p.ldo + n] =
          gemm_epilogue<T>(acc[r], p.has_bias, p.alpha, p.beta, bj);
    }
  }
}

template <typename T, bool B_NK>
static int launch_typed(const GemmArgs& g, cudaStream_t stream) {
  Params p;
  p.a = g.a;
  p.lda = g.lda;
  p.b = g.b;
  p.ldb = g.ldb;
  p.bias = g.bias;
  p.out = g.out;
  p.ldo = g.ldo;
  p.M = static_cast<int>(g.M);
  p.N = static_cast<int>(g.N);
  p.K = static_cast<int>(g.K);
  p.alpha = g.alpha;
  p.beta = g.beta;
  p.has_bias = g.bias != nullptr;
  if (B_NK && g.M <= ROWS_MAX_M) {
    // few rows: one warp per column (same per-element arithmetic as the tiled kernel)
    const int maxm = g.M <= 32 ? 32 : 64;
    const int64_t blocks = (g.N + rows_warps(maxm) - 1) / rows_warps(maxm);
    if (blocks > 0x7fffffffLL) return set_error(BI_ERR_UNSUPPORTED, "N too large");
    const size_t es = sizeof(T);
    const bool vec = (reinterpret_cast<uintptr_t>(g.a) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(g.b) % 16 == 0) && (g.lda * es) % 16 == 0 &&
                     (g.ldb * es) % 16 == 0;
    const unsigned nb = static_cast<unsigned>(blocks);
    if (maxm == 32) {
      constexpr int nt = 32 * rows_warps(32);
      if (vec) gemm_simt_rows_kernel<T, true, 32><<<nb, nt, 0, stream>>>(p);
      else gemm_simt_rows_kernel<T, false, 32><<<nb, nt, 0, stream>>>(p);
    } else {
      constexpr int nt = 32 * rows_warps(64);
      if (vec) gemm_simt_rows_kernel<T, true, 64><<<nb, nt, 0, stream>>>(p);
      else gemm_simt_rows_kernel<T, false, 64><<<nb, nt, 0, stream>>>(p);
    }
    return cuda_status(cudaGetLastError(), "gemm_simt rows launch");
  }
  const int64_t gy = (g.M + BM - 1) / BM;
  const int64_t gx = (g.N + BN - 1) / BN;
  if (gy > 65535) return set_error(BI_ERR_UNSUPPORTED, "M too large for the CUDA-core route");
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  gemm_simt_kernel<T, B_NK><<<grid, NUM_THREADS, 0, stream>>>(p);
  return cuda_status(cudaGetLastError(), "gemm_simt launch");
}

}  // namespace simt

int launch_gemm_simt(const GemmArgs& g, cudaStream_t stream) {
  if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX) {
    return set_error(BI_ERR_UNSUPPORTED, "dimensions above 2^31 are not supported");
  }
  switch (g.dtype) {
    case BI_F32:
      return g.b_is_nk ? simt::launch_typed<float, true>(g, stream)
                       : simt::launch_typed<float, false>(g, stream);
    case BI_F16:
      return g.b_is_nk ? simt::launch_typed<__half, true>(g, stream)
                       : simt::launch_typed<__half, false>(g, stream);
    case BI_BF16:
      return g.b_is_nk ? simt::launch_typed<__nv_bfloat16, true>(g, stream)
                       : simt::launch_typed<__nv_bfloat16, false>(g, stream);
    default:
      return set_error(BI_ERR_INVALID, "unknown dtype %d", g.dtype);
  }
}

}  // namespace bi
