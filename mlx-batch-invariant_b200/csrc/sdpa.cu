// Batch-invariant single-pass scaled dot-product attention.
//
// Fold (the algorithm of mlx_batch_invariant/_attention.py:32-149, restated): one
// CTA owns one query row s of one (batch b, head h) -- or of a small group of query
// heads that share a KV head, which changes only which CTA does the work -- and the
// whole reduction over the N keys.  Key i always folds into partial p = i % 32.
// Each partial keeps an fp32 online-softmax state (running max m, denominator l,
// numerator o[V]); the 32 partials are then combined in the fixed order p = 0..31.
// Nothing depends on B, H, qL or on the other rows in flight: there is no split-KV,
// no second pass and no route switch, so a token's output has the same bits in
// decode and in any chunked prefill, and an extra masked key is a no-op.
//
// B200 mapping:
//   * K and V rows of the KV head are streamed through a ring of shared-memory
//     stages with 1-D bulk copies (cp.async.bulk, mbarrier completion), 32 keys per
//     stage -- one key per partial -- so the bytes in flight do not depend on
//     registers.
//   * A partial is LP consecutive threads; each holds D/LP elements of q, k, v and o
//     (16-byte vectors where the row allows).  The q.k dot product is a sequential
//     fmaf over the thread's elements followed by a fixed xor-butterfly over the LP
//     threads, which leaves the identical sum in every thread of the partial.
//   * Online-softmax update per visible key (i = key, h = head):
//         m' = max(m, score);  f = exp(m - m');  e = exp(score - m')
//         l  = fmaf(l, f, e);  o[j] = fmaf(e, v[j], o[j] * f);  m = m'
//     When m' == m the multiply by f = exp(0) = 1 is skipped (bit-identical).
//   * Combine: M = max_p m_p; f_p = exp(m_p - M); l = sum_p fmaf(l_p, f_p, .);
//     out[j] = (sum_p fmaf(o_p[j], f_p, .)) / l, or 0 when l == 0 (fully masked).
#include "common.cuh"
#include "internal.h"

namespace bi {
namespace sdpa {

constexpr int PARTIALS = 32;  // also the key stride of the walk (reference BN = 32)

__device__ unsigned g_error_word = 0;

struct Params {
  const void* q;
  int64_t qs0, qs1, qs2;
  const void* k;
  int64_t ks0, ks1;
  const void* v;
  int64_t vs0, vs1;
  const void* mask;
  int64_t ms0, ms1, ms2;
  int mask_mode;
  int64_t causal_offset;
  const void* sinks;
  float scale;
  int B, H, Hkv, qL, N;
  void* out;
  int64_t os0, os1, os2;
};

// Loads E contiguous elements of type T starting at `src` (aligned to the largest
// power-of-two divisor of E*sizeof(T), at most 16 bytes) and widens them to fp32.
template <typename T, int E>
__device__ __forceinline__ void load_vec(const T* src, float (&dst)[E]) {
  constexpr int BYTES = E * static_cast<int>(sizeof(T));
  constexpr int W = (BYTES % 16 == 0) ? 16 : (BYTES % 8 == 0) ? 8 : (BYTES % 4 == 0) ? 4 : 2;
  constexpr int PER = W / static_cast<int>(sizeof(T)) > 0 ? W / static_cast<int>(sizeof(T)) : 1;
  if constexpr (W >= static_cast<int>(sizeof(T))) {
#pragma unroll
    for (int c = 0; c < E / PER; ++c) {
      T tmp[PER];
      if constexpr (W == 16) {
        *reinterpret_cast<uint4*>(tmp) = *reinterpret_cast<const uint4*>(src + c * PER);
      } else if constexpr (W == 8) {
        *reinterpret_cast<uint2*>(tmp) = *reinterpret_cast<const uint2*>(src + c * PER);
      } else if constexpr (W == 4) {
        *reinterpret_cast<uint32_t*>(tmp) = *reinterpret_cast<const uint32_t*>(src + c * PER);
      } else {
        tmp[0] = src[c * PER];
      }
#pragma unroll
      for (int u = 0; u < PER; ++u) dst[c * PER + u] = to_f32(tmp[u]);
    }
  }
}

template <typename T, int D, int LP, int HG, int STAGES>
__global__ void __launch_bounds__(PARTIALS * LP) sdpa_kernel(const Params p) {
  constexpr int NT = PARTIALS * LP;
  constexpr int E = D / LP;  // elements of q/k/v/o per thread
  constexpr int ROW_BYTES = D * static_cast<int>(sizeof(T));
  constexpr int STAGE_ELEMS = PARTIALS * D;
  static_assert(D % LP == 0, "D must split evenly over the partial's threads");
  static_assert(32 % LP == 0, "a partial must not straddle warps");

  extern __shared__ __align__(128) uint8_t smem[];
  T* sK = reinterpret_cast<T*>(smem);
  T* sV = sK + STAGES * STAGE_ELEMS;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * STAGES * PARTIALS * ROW_BYTES);
  float* comb_m = reinterpret_cast<float*>(full + STAGES);  // [PARTIALS]
  float* comb_l = comb_m + PARTIALS;                         // [PARTIALS]
  float* comb_o = reinterpret_cast<float*>(smem);            // [PARTIALS][D], after the walk

  const int tid = threadIdx.x;
  const int part = tid / LP;
  const int sub = tid % LP;

  // Block -> (b, head group, s); s fastest.
  const int groups = p.H / HG;
  int idx = blockIdx.x;
  const int s = idx % p.qL;
  idx /= p.qL;
  const int hg = idx % groups;
  const int b = idx / groups;
  const int h0 = hg * HG;
  const int kvh = h0 / (p.H / p.Hkv);

  int64_t kmax = p.N;
  if (p.mask_mode == 1) {
    const int64_t last = p.causal_offset + s;  // last visible key
    kmax = last < 0 ? 0 : (last + 1 < p.N ? last + 1 : p.N);
  }
  const int nblocks = static_cast<int>((kmax + PARTIALS - 1) / PARTIALS);

  const T* Q = static_cast<const T*>(p.q);
  const T* Kb = static_cast<const T*>(p.k) + static_cast<int64_t>(b) * p.ks0 +
                static_cast<int64_t>(kvh) * p.ks1;
  const T* Vb = static_cast<const T*>(p.v) + static_cast<int64_t>(b) * p.vs0 +
                static_cast<int64_t>(kvh) * p.vs1;
  const T* Mk = static_cast<const T*>(p.mask);
  const T* Sk = static_cast<const T*>(p.sinks);

  float qv[HG][E], o[HG][E], m[HG], l[HG];
#pragma unroll
  for (int h = 0; h < HG; ++h) {
    const T* qrow = Q + static_cast<int64_t>(b) * p.qs0 + static_cast<int64_t>(h0 + h) * p.qs1 +
                    static_cast<int64_t>(s) * p.qs2 + sub * E;
    float tmp[E];
    load_vec<T, E>(qrow, tmp);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      qv[h][e] = __fmul_rn(p.scale, tmp[e]);
      o[h][e] = 0.f;
    }
    // Lowest finite float, not -inf, so a fully masked partial stays NaN-free.
    m[h] = -3.40282347e+38f;
    l[h] = 0.f;
    if (Sk != nullptr && part == 0) {
      m[h] = to_f32(Sk[h0 + h]);
      l[h] = 1.f;
    }
  }

  if (tid == 0) {
    for (int st = 0; st < STAGES; ++st) mbar_init(&full[st], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int blk) {
    const int st = blk % STAGES;
    const int64_t i0 = static_cast<int64_t>(blk) * PARTIALS;
    const int64_t rows = (kmax - i0) < PARTIALS ? (kmax - i0) : PARTIALS;
    const uint32_t bytes = static_cast<uint32_t>(rows) * ROW_BYTES;
    mbar_arrive_expect_tx(&full[st], 2 * bytes);
    bulk_load(sK + st * STAGE_ELEMS, Kb + i0 * D, bytes, &full[st]);
    bulk_load(sV + st * STAGE_ELEMS, Vb + i0 * D, bytes, &full[st]);
  };

  int issued = 0;
  if (tid == 0) {
    for (; issued < STAGES && issued < nblocks; ++issued) issue(issued);
  }

  bool aborted = false;
  for (int t = 0; t < nblocks; ++t) {
    const int st = t % STAGES;
    const bool ok = mbar_wait(&full[st], static_cast<uint32_t>((t / STAGES) & 1), nullptr);
    if (!__syncthreads_and(ok)) {
      aborted = true;
      break;
    }
    // Every thread has finished block t-1, so its stage may be refilled.
    if (tid == 0 && t >= 1 && issued < nblocks) {
      issue(issued);
      ++issued;
    }
    const int64_t i = static_cast<int64_t>(t) * PARTIALS + part;
    const bool in_range = i < kmax;
    float kf[E], vf[E];
    load_vec<T, E>(sK + st * STAGE_ELEMS + part * D + sub * E, kf);
    load_vec<T, E>(sV + st * STAGE_ELEMS + part * D + sub * E, vf);
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      float bias = 0.f;
      bool use = in_range;
      if (p.mask_mode == 2 && in_range) {
        bias = to_f32(Mk[static_cast<int64_t>(b) * p.ms0 + static_cast<int64_t>(h0 + h) * p.ms1 +
                         static_cast<int64_t>(s) * p.ms2 + i]);
        use = bias > -3.0e38f;
      }
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) dot = __fmaf_rn(qv[h][e], kf[e], dot);
#pragma unroll
      for (int off = LP / 2; off >= 1; off >>= 1) {
        dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, off));
      }
      if (use) {
        const float score = __fadd_rn(dot, bias);
        if (score > m[h]) {
          const float f = expf(__fsub_rn(m[h], score));
          m[h] = score;
          // e = exp(score - m') = exp(0) = 1
          l[h] = __fmaf_rn(l[h], f, 1.0f);
#pragma unroll
          for (int e = 0; e < E; ++e) o[h][e] = __fmaf_rn(1.0f, vf[e], __fmul_rn(o[h][e], f));
        } else {
          const float ex = expf(__fsub_rn(score, m[h]));
          l[h] = __fadd_rn(l[h], ex);
#pragma unroll
          for (int e = 0; e < E; ++e) o[h][e] = __fmaf_rn(ex, vf[e], o[h][e]);
        }
      }
    }
  }

  if (aborted) {
    if (tid == 0) {
      record_error(&g_error_word, (1u << 8) | kErrReasonTimeout);
      // Drain: wait (bounded) for the copies still in flight before leaving.
      for (int blk = 0; blk < issued; ++blk) {
        mbar_wait(&full[blk % STAGES], static_cast<uint32_t>((blk / STAGES) & 1), nullptr);
      }
    }
    return;
  }

  // ---- combine the 32 partials, one head at a time ----
  T* O = static_cast<T*>(p.out);
#pragma unroll
  for (int h = 0; h < HG; ++h) {
    __syncthreads();  // stage buffers (and the previous head's combine) are free
#pragma unroll
    for (int e = 0; e < E; ++e) comb_o[part * D + sub * E + e] = o[h][e];
    if (sub == 0) {
      comb_m[part] = m[h];
      comb_l[part] = l[h];
    }
    __syncthreads();
    for (int j = tid; j < D; j += NT) {
      float mx = comb_m[0];
#pragma unroll
      for (int q = 1; q < PARTIALS; ++q) mx = fmaxf(mx, comb_m[q]);
      float lsum = 0.f, acc = 0.f;
#pragma unroll 4
      for (int q = 0; q < PARTIALS; ++q) {
        const float f = expf(__fsub_rn(comb_m[q], mx));
        lsum = __fmaf_rn(comb_l[q], f, lsum);
        acc = __fmaf_rn(comb_o[q * D + j], f, acc);
      }
      const float res = lsum == 0.f ? acc : __fdiv_rn(acc, lsum);
      O[static_cast<int64_t>(b) * p.os0 + static_cast<int64_t>(h0 + h) * p.os1 +
        static_cast<int64_t>(s) * p.os2 + j] = from_f32<T>(res);
    }
  }
}

// Threads per partial: 16-byte vectors per thread where the row allows, a power of
// two that divides D, at most 32.  A function of (D, dtype) only.
template <typename T>
constexpr int lanes_for(int D) {
  int lp = (D * static_cast<int>(sizeof(T))) / 16;
  if (lp > 32) lp = 32;
  int p2 = 1;
  while (p2 * 2 <= lp) p2 *= 2;
  while (p2 > 1 && D % p2 != 0) p2 /= 2;
  return p2;
}

template <typename T, int D>
constexpr int stages_for() {
  constexpr int pair = 2 * PARTIALS * D * static_cast<int>(sizeof(T));
  constexpr int s = (96 * 1024) / pair;
  return s < 2 ? 2 : (s > 4 ? 4 : s);
}

template <typename T, int D>
constexpr int max_heads_per_cta() {
  constexpr int LP = lanes_for<T>(D);
  constexpr int E = D / LP;
  constexpr int budget = (PARTIALS * LP == 1024) ? 32 : 64;  // registers for q and o
  return (8 * E <= budget) ? 4 : (4 * E <= budget) ? 2 : 1;
}

template <typename T, int D, int HG>
static int launch_hg(const Params& p, int64_t blocks, cudaStream_t stream) {
  constexpr int LP = lanes_for<T>(D);
  constexpr int S = stages_for<T, D>();
  constexpr int NT = PARTIALS * LP;
  constexpr int smem = 2 * S * PARTIALS * D * static_cast<int>(sizeof(T)) + S * 8 +
                       2 * PARTIALS * 4;
  static_assert(PARTIALS * D * 4 <= 2 * S * PARTIALS * D * static_cast<int>(sizeof(T)),
                "combine buffer must fit in the stage ring");
  auto kern = sdpa_kernel<T, D, LP, HG, S>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(sdpa)");
  if (blocks > 0x7fffffffLL) return set_error(BI_ERR_UNSUPPORTED, "too many attention rows");
  kern<<<static_cast<unsigned>(blocks), NT, smem, stream>>>(p);
  return cuda_status(cudaGetLastError(), "sdpa launch");
}

template <typename T, int D>
static int launch_d(const SdpaArgs& a, const Params& p, cudaStream_t stream) {
  constexpr int HGMAX = max_heads_per_cta<T, D>();
  const int64_t G = a.H / a.Hkv;
  // Heads per CTA: the largest of {4, 2, 1} within the register budget that divides
  // the GQA factor.  It decides which CTA computes a row, never the row's arithmetic.
  int hg = 1;
  if (HGMAX >= 4 && G % 4 == 0) hg = 4;
  else if (HGMAX >= 2 && G % 2 == 0) hg = 2;
  const int64_t blocks = a.B * (a.H / hg) * a.qL;
  switch (hg) {
    case 4:
      if constexpr (HGMAX >= 4) return launch_hg<T, D, 4>(p, blocks, stream);
      break;
    case 2:
      if constexpr (HGMAX >= 2) return launch_hg<T, D, 2>(p, blocks, stream);
      break;
    default:
      break;
  }
  return launch_hg<T, D, 1>(p, blocks, stream);
}

template <typename T>
static int launch_t(const SdpaArgs& a, const Params& p, cudaStream_t stream) {
  switch (a.D) {
    case 32: return launch_d<T, 32>(a, p, stream);
    case 64: return launch_d<T, 64>(a, p, stream);
    case 96: return launch_d<T, 96>(a, p, stream);
    case 128: return launch_d<T, 128>(a, p, stream);
    case 160: return launch_d<T, 160>(a, p, stream);
    case 192: return launch_d<T, 192>(a, p, stream);
    case 224: return launch_d<T, 224>(a, p, stream);
    case 256: return launch_d<T, 256>(a, p, stream);
    default:
      return set_error(BI_ERR_UNSUPPORTED, "head dim %lld is not built (multiples of 32 up to 256)",
                       static_cast<long long>(a.D));
  }
}

}  // namespace sdpa

int launch_sdpa(const SdpaArgs& a, cudaStream_t stream) {
  sdpa::Params p;
  p.q = a.q;
  p.qs0 = a.qs[0];
  p.qs1 = a.qs[1];
  p.qs2 = a.qs[2];
  p.k = a.k;
  p.ks0 = a.ks[0];
  p.ks1 = a.ks[1];
  p.v = a.v;
  p.vs0 = a.vs[0];
  p.vs1 = a.vs[1];
  p.mask = a.mask;
  p.ms0 = a.ms[0];
  p.ms1 = a.ms[1];
  p.ms2 = a.ms[2];
  p.mask_mode = a.mask_mode;
  p.causal_offset = a.causal_offset;
  p.sinks = a.sinks;
  p.scale = a.scale;
  p.B = static_cast<int>(a.B);
  p.H = static_cast<int>(a.H);
  p.Hkv = static_cast<int>(a.Hkv);
  p.qL = static_cast<int>(a.qL);
  p.N = static_cast<int>(a.N);
  p.out = a.out;
  p.os0 = a.os[0];
  p.os1 = a.os[1];
  p.os2 = a.os[2];
  switch (a.dtype) {
    case BI_F32: return sdpa::launch_t<float>(a, p, stream);
    case BI_F16: return sdpa::launch_t<__half>(a, p, stream);
    case BI_BF16: return sdpa::launch_t<__nv_bfloat16>(a, p, stream);
    default: return set_error(BI_ERR_INVALID, "unknown dtype %d", a.dtype);
  }
}

unsigned read_error_sdpa(bool clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, sdpa::g_error_word, sizeof(v));
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(sdpa::g_error_word, &z, sizeof(z));
  }
  return v;
}

}  // namespace bi
