// Batch-invariant single-pass scaled dot-product attention.
//
// Fold (the algorithm of mlx_batch_invariant/_attention.py:32-149, restated): one
// CTA owns one query row s of one (batch b, head h) -- or of a small group of query
// heads that share a KV head, which changes only which CTA does the work -- and the
// whole reduction over the N keys.  Key i always folds into partial p = i % 32.
// Each partial keeps an fp32 online-softmax state (running max m, denominator l,
// numerator o[V]); the 32 partials are then combined in the fixed order p = 0..31.
// Nothing depends on B, qL, N or on the other rows in flight: there is no split-KV,
// no second pass, and the route (the CUDA-core kernel here, the GQA kernel further down
// -- q.k on the tensor cores, fold and P.V in fp32 -- for 16-bit data with D = 64 / 128
// and GQA groups of 4k heads, or the generic kernel for other head dims) is a function
// of the model's shapes alone, so a token's output has the same bits in decode and in
// any chunked prefill, and an extra masked key is a no-op.
//
// B200 mapping:
//   * K and V rows of the KV head are streamed through a ring of shared-memory
//     stages with 1-D bulk copies (cp.async.bulk, one mbarrier per stage), ROWS keys
//     per partial per stage, so the bytes in flight do not depend on registers; the
//     last warp to finish a stage refills it, so no CTA-wide barrier sits in the loop.
//   * A partial is LP consecutive threads, each holding E = D/LP elements of q, k, v
//     and o (32 bytes of a key row per thread, as interleaved 16-byte vectors so a
//     quarter warp reads distinct banks); LP is a function of (D, dtype) only.
//   * Arithmetic uses Blackwell's packed fp32x2 FMA/MUL (fma.rn.f32x2), which rounds
//     each lane exactly like fmaf.  The q.k dot product of a thread runs four fp32
//     chains (its k-th element goes to chain (k/2 % 2)*2 + k%2), summed as
//     (c0 + c1) + (c2 + c3); a fixed
//     xor-butterfly over the LP threads sums it.  The CTA's heads share one butterfly
//     (reduce_heads): each thread ends with one head's score and runs that head's
//     scalar softmax step; the weights reach the other threads by shuffle.
//   * Online-softmax update per visible key (h = head):
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

// Key rows per partial in one shared-memory stage (stage = PARTIALS * ROWS keys), at
// most this many; it changes how keys are staged, never the fold.
#ifndef BI_SDPA_ROWS_PER_STAGE
#define BI_SDPA_ROWS_PER_STAGE 2
#endif
// Registers per thread available for the q and o slices of the CTA's heads.
#ifndef BI_SDPA_REG_BUDGET
#define BI_SDPA_REG_BUDGET 64
#endif

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
  int D, V;  // head dims (the generic kernel reads them; the others have them built in)
  void* out;
  int64_t os0, os1, os2;
};

// ---- packed fp32x2 arithmetic (each lane rounded as the scalar op) ----
struct f2 {
  uint64_t r;
};
__device__ __forceinline__ f2 pack2(float lo, float hi) {
  return f2{static_cast<uint64_t>(__float_as_uint(lo)) |
            (static_cast<uint64_t>(__float_as_uint(hi)) << 32)};
}
__device__ __forceinline__ float lo_of(f2 a) { return __uint_as_float(static_cast<uint32_t>(a.r)); }
__device__ __forceinline__ float hi_of(f2 a) {
  return __uint_as_float(static_cast<uint32_t>(a.r >> 32));
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d.r) : "l"(a.r), "l"(b.r), "l"(c.r));
  return d;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d.r) : "l"(a.r), "l"(b.r));
  return d;
}

// A thread's share of a D-element row: E elements taken as NV vectors of W bytes
// (W = 16, 8 or 4, whichever divides E*sizeof(T)), vector c of thread `sub` starting
// at element (c*LP + sub)*PER.  Interleaving the threads' vectors keeps each quarter
// warp's shared-memory reads on distinct banks.
template <typename T, int E>
struct RowSlice {
  static constexpr int BYTES = E * static_cast<int>(sizeof(T));
  static constexpr int W = (BYTES % 16 == 0) ? 16 : (BYTES % 8 == 0) ? 8 : 4;
  static constexpr int PER = W / static_cast<int>(sizeof(T));  // elements per vector
  static constexpr int NV = E / PER;                           // vectors per thread
  static constexpr int WORDS = W / 4;
};

// Element index (within the row) of the thread's k-th element.
template <typename T, int E, int LP>
__device__ __forceinline__ int slice_elem(int sub, int k) {
  using RS = RowSlice<T, E>;
  return ((k / RS::PER) * LP + sub) * RS::PER + k % RS::PER;
}

// Loads the thread's slice of a row (see RowSlice) and widens it to E/2 packed fp32
// pairs (the thread's element 2j in the low half, 2j+1 in the high half).
template <typename T, int E, int LP>
__device__ __forceinline__ void load_slice(const T* row, int sub, f2 (&dst)[E / 2]) {
  using RS = RowSlice<T, E>;
  constexpr int WORDS = RS::WORDS;
#pragma unroll
  for (int c = 0; c < RS::NV; ++c) {
    const uint32_t* s =
        reinterpret_cast<const uint32_t*>(row + (c * LP + sub) * RS::PER);
    uint32_t w[WORDS];
    if constexpr (RS::W == 16) {
      const uint4 u = *reinterpret_cast<const uint4*>(s);
      w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
    } else if constexpr (RS::W == 8) {
      const uint2 u = *reinterpret_cast<const uint2*>(s);
      w[0] = u.x; w[1] = u.y;
    } else {
      w[0] = s[0];
    }
#pragma unroll
    for (int i = 0; i < WORDS; ++i) {
      if constexpr (sizeof(T) == 4) {
        // fp32: two words make one pair
        if (i % 2 == 1) dst[(c * WORDS + i) / 2] = f2{static_cast<uint64_t>(w[i - 1]) |
                                                      (static_cast<uint64_t>(w[i]) << 32)};
      } else if constexpr (dtype_of<T>::value == 2) {
        // bf16 pair in one word: widening is a shift / mask
        dst[c * WORDS + i] = f2{static_cast<uint64_t>(w[i] << 16) |
                                (static_cast<uint64_t>(w[i] & 0xffff0000u) << 32)};
      } else {
        const float2 fl = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        dst[c * WORDS + i] = pack2(fl.x, fl.y);
      }
    }
  }
}

// Head whose score thread `sub` holds after the transposed butterfly below.
template <int LP, int HG>
__device__ __forceinline__ int own_head(int sub) {
  int h = 0, nv = HG;
#pragma unroll
  for (int off = LP / 2; off >= 1; off >>= 1) {
    if (nv > 1) {
      nv >>= 1;
      if (sub & off) h += nv;
    }
  }
  return h;
}

// Sums each head's per-thread partial dot over the LP threads of a partial with the
// xor-butterfly (offsets LP/2, ..., 1).  While more than one head is in flight, each
// level halves the heads a thread carries (the partner of a pair keeps the other
// half), so the sum of every head is formed by exactly the additions of a plain
// butterfly for that head -- a+b and b+a being the same fp32 value -- and thread
// `sub` ends with the total of head own_head(sub).
template <int LP, int HG>
__device__ __forceinline__ float reduce_heads(float (&v)[HG], int sub) {
  int nv = HG;
#pragma unroll
  for (int off = LP / 2; off >= 1; off >>= 1) {
    if (nv > 1) {
      const int half = nv >> 1;
      const bool upper = (sub & off) != 0;
#pragma unroll
      for (int j = 0; j < HG / 2; ++j) {
        if (j < half) {
          const float send = upper ? v[j] : v[j + half];
          const float keep = upper ? v[j + half] : v[j];
          v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
        }
      }
      nv = half;
    } else {
      v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], off));
    }
  }
  return v[0];
}

// Combine weights of one head, computed once by one warp (lane q = partial q): the
// largest running max M over the 32 partials, f_q = exp(m_q - M) (written over m_q),
// and the denominator sum_q fmaf(l_q, f_q, .) in the order q = 0..31.  The output
// loop then only runs its own ordered fmaf chain over the stored f_q.
__device__ __forceinline__ float combine_weights(float* cm, const float* cl, int lane) {
  const float mq = cm[lane];
  float mx = mq;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float fq = expf(__fsub_rn(mq, mx));
  __syncwarp();
  cm[lane] = fq;
  __syncwarp();
  float lsum = 0.f;
  if (lane == 0) {
#pragma unroll 8
    for (int q = 0; q < PARTIALS; ++q) lsum = __fmaf_rn(cl[q], cm[q], lsum);
  }
  return __shfl_sync(0xffffffffu, lsum, 0);
}

#ifndef BI_SDPA_MIN_BLOCKS
#define BI_SDPA_MIN_BLOCKS 1
#endif

template <typename T, int D, int LP, int HG, int STAGES, int ROWS>
__global__ void __launch_bounds__(PARTIALS * LP, (PARTIALS * LP <= 256 ? BI_SDPA_MIN_BLOCKS : 1))
    sdpa_kernel(const Params p) {
  constexpr int NT = PARTIALS * LP;
  constexpr int NW = NT / 32;  // warps
  constexpr int E = D / LP;  // elements of q/k/v/o per thread
  constexpr int E2 = E / 2;
  constexpr int ROW_BYTES = D * static_cast<int>(sizeof(T));
  constexpr int KEYS = PARTIALS * ROWS;  // keys per stage
  constexpr int STAGE_ELEMS = KEYS * D;
  static_assert(D % LP == 0 && E % 2 == 0, "D must split evenly into pairs per thread");
  static_assert(32 % LP == 0, "a partial must not straddle warps");
  static_assert(HG <= LP, "each head's softmax state needs a thread of its own");

  extern __shared__ __align__(128) uint8_t smem[];
  T* sK = reinterpret_cast<T*>(smem);
  T* sV = sK + STAGES * STAGE_ELEMS;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * STAGES * KEYS * ROW_BYTES);
  int* done_count = reinterpret_cast<int*>(full + STAGES);          // [STAGES]
  int* issued_count = done_count + STAGES;
  volatile int* abort_flag = issued_count + 1;
  float* comb_m = reinterpret_cast<float*>(done_count + STAGES + 4);  // [PARTIALS]
  float* comb_l = comb_m + PARTIALS;                         // [PARTIALS + 1]
  float* comb_o = reinterpret_cast<float*>(smem);            // [PARTIALS][D], after the walk

  const int tid = threadIdx.x;
  const int part = tid / LP;
  const int sub = tid % LP;
  const int lane = tid & 31;
  const int part_lane0 = lane & ~(LP - 1);  // first lane of this partial in the warp
  const int my_head = own_head<LP, HG>(sub);

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
  const int nblocks = static_cast<int>((kmax + KEYS - 1) / KEYS);

  const T* Q = static_cast<const T*>(p.q);
  const T* Kb = static_cast<const T*>(p.k) + static_cast<int64_t>(b) * p.ks0 +
                static_cast<int64_t>(kvh) * p.ks1;
  const T* Vb = static_cast<const T*>(p.v) + static_cast<int64_t>(b) * p.vs0 +
                static_cast<int64_t>(kvh) * p.vs1;
  const T* Mk = static_cast<const T*>(p.mask);
  const T* mrow = Mk == nullptr ? nullptr
                                : Mk + static_cast<int64_t>(b) * p.ms0 +
                                      static_cast<int64_t>(h0 + my_head) * p.ms1 +
                                      static_cast<int64_t>(s) * p.ms2;
  const T* Sk = static_cast<const T*>(p.sinks);

  f2 qv[HG][E2], o[HG][E2];
#pragma unroll
  for (int h = 0; h < HG; ++h) {
    const T* qrow = Q + static_cast<int64_t>(b) * p.qs0 + static_cast<int64_t>(h0 + h) * p.qs1 +
                    static_cast<int64_t>(s) * p.qs2;
    f2 tmp[E2];
    load_slice<T, E, LP>(qrow, sub, tmp);
    const f2 sc = pack2(p.scale, p.scale);
#pragma unroll
    for (int c = 0; c < E2; ++c) {
      qv[h][c] = mul2(sc, tmp[c]);
      o[h][c] = f2{0};
    }
  }
  // Softmax state of head my_head for this partial.  Lowest finite float, not -inf,
  // so a fully masked partial stays NaN-free; a sink seeds partial 0.
  float m = -3.40282347e+38f;
  float l = 0.f;
  if (Sk != nullptr && part == 0) {
    m = to_f32(Sk[h0 + my_head]);
    l = 1.f;
  }

  auto issue = [&](int blk) {
    const int st = blk % STAGES;
    const int64_t i0 = static_cast<int64_t>(blk) * KEYS;
    const int64_t rows = (kmax - i0) < KEYS ? (kmax - i0) : KEYS;
    const uint32_t bytes = static_cast<uint32_t>(rows) * ROW_BYTES;
    mbar_arrive_expect_tx(&full[st], 2 * bytes);
    bulk_load(sK + st * STAGE_ELEMS, Kb + i0 * D, bytes, &full[st]);
    bulk_load(sV + st * STAGE_ELEMS, Vb + i0 * D, bytes, &full[st]);
  };

  if (tid == 0) {
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&full[st], 1);
      done_count[st] = 0;
    }
    *abort_flag = 0;
    fence_barrier_init();
    int n0 = 0;
    for (; n0 < STAGES && n0 < nblocks; ++n0) issue(n0);
    *issued_count = n0;
  }
  __syncthreads();

  bool aborted = false;
  for (int t = 0; t < nblocks; ++t) {
    const int st = t % STAGES;
    bool ok = mbar_wait(&full[st], static_cast<uint32_t>((t / STAGES) & 1), abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) {
      if (lane == 0) {
        *abort_flag = 1;
        record_error(&g_error_word, (1u << 8) | kErrReasonTimeout);
      }
      aborted = true;
      break;
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      // key i = t*KEYS + r*PARTIALS + part: partial `part` sees its keys in order
      const int row = r * PARTIALS + part;
      const int64_t i = static_cast<int64_t>(t) * KEYS + row;
      const bool in_range = i < kmax;
      f2 kf[E2];
      load_slice<T, E, LP>(sK + st * STAGE_ELEMS + row * D, sub, kf);
      float dots[HG];
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        // four fp32 chains: pairs c even -> acc[0], c odd -> acc[1]
        f2 acc[2] = {f2{0}, f2{0}};
#pragma unroll
        for (int c = 0; c < E2; ++c) acc[c & 1] = fma2(qv[h][c], kf[c], acc[c & 1]);
        dots[h] = __fadd_rn(__fadd_rn(lo_of(acc[0]), hi_of(acc[0])),
                            __fadd_rn(lo_of(acc[1]), hi_of(acc[1])));
      }
      const float dot = reduce_heads<LP, HG>(dots, sub);

      // Scalar online-softmax step for head my_head.  ex < 0 marks a skipped key.
      float bias = 0.f;
      bool use = in_range;
      if (p.mask_mode == 2 && in_range) {
        bias = to_f32(mrow[i]);
        use = bias > -3.0e38f;
      }
      float ex = -1.f, f = 1.f;
      if (use) {
        const float score = __fadd_rn(dot, bias);
        if (score > m) {
          f = expf(__fsub_rn(m, score));
          m = score;
          ex = 1.0f;  // exp(score - m') = exp(0)
          l = __fmaf_rn(l, f, 1.0f);
        } else {
          ex = expf(__fsub_rn(score, m));
          l = __fadd_rn(l, ex);
        }
      }
      const bool any_rescale = __any_sync(0xffffffffu, f != 1.0f);

      f2 vf[E2];
      load_slice<T, E, LP>(sV + st * STAGE_ELEMS + row * D, sub, vf);
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        const int src = part_lane0 + (HG == 1 ? sub : h * (LP / HG));
        const float eh = HG == 1 ? ex : __shfl_sync(0xffffffffu, ex, src);
        float fh = 1.f;
        if (any_rescale) fh = HG == 1 ? f : __shfl_sync(0xffffffffu, f, src);
        if (!(eh < 0.f)) {
          if (fh != 1.0f) {
            const f2 f_2 = pack2(fh, fh);
#pragma unroll
            for (int c = 0; c < E2; ++c) o[h][c] = mul2(o[h][c], f_2);
          }
          const f2 e_2 = pack2(eh, eh);
#pragma unroll
          for (int c = 0; c < E2; ++c) o[h][c] = fma2(e_2, vf[c], o[h][c]);
        }
      }
    }
    // The last warp to finish with this stage refills it with block t + STAGES; no
    // warp waits for another.
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&done_count[st], 1) == NW - 1) {
        __threadfence_block();
        done_count[st] = 0;
        if (t + STAGES < nblocks && !*abort_flag) {
          fence_proxy_async_smem();
          issue(t + STAGES);
          atomicMax(issued_count, t + STAGES + 1);
        }
      }
    }
  }
  if (__syncthreads_or(aborted)) {
    if (tid == 0) {
      // Drain: wait (bounded) for the last fill of every stage still in flight.
      const int issued = *issued_count;
      for (int blk = issued - STAGES < 0 ? 0 : issued - STAGES; blk < issued; ++blk) {
        mbar_wait(&full[blk % STAGES], static_cast<uint32_t>((blk / STAGES) & 1), nullptr);
      }
    }
    return;
  }
  __syncthreads();

  // ---- combine the 32 partials, one head at a time ----
  T* O = static_cast<T*>(p.out);
#pragma unroll
  for (int h = 0; h < HG; ++h) {
    __syncthreads();  // stage buffers (and the previous head's combine) are free
#pragma unroll
    for (int c = 0; c < E2; ++c) {
      *reinterpret_cast<float2*>(&comb_o[part * D + slice_elem<T, E, LP>(sub, 2 * c)]) =
          make_float2(lo_of(o[h][c]), hi_of(o[h][c]));
    }
    if (sub == h * (LP / HG)) {
      comb_m[part] = m;
      comb_l[part] = l;
    }
    __syncthreads();
    if (tid < 32) {
      const float ls = combine_weights(comb_m, comb_l, tid);  // comb_m now holds f_q
      if (tid == 0) comb_l[PARTIALS] = ls;
    }
    __syncthreads();
    const float lsum = comb_l[PARTIALS];
    for (int j = tid; j < D; j += NT) {
      float acc = 0.f;
#pragma unroll 8
      for (int q = 0; q < PARTIALS; ++q) acc = __fmaf_rn(comb_o[q * D + j], comb_m[q], acc);
      const float res = lsum == 0.f ? acc : __fdiv_rn(acc, lsum);
      O[static_cast<int64_t>(b) * p.os0 + static_cast<int64_t>(h0 + h) * p.os1 +
        static_cast<int64_t>(s) * p.os2 + j] = from_f32<T>(res);
    }
  }
}


// ---------------------------------------------------------------------------
// Generic head dims: D != V, or either above 256 (multiples of 32; D, V <= 640 for
// 16-bit types -- MLA's 576 / 512 among them -- and D, V <= 384, D + V <= 768 for
// float32).  The same fold as sdpa_kernel, one query
// head per CTA, with the head dims known only at run time:
//   * a partial is 16 threads; thread `sub` holds elements (2c*16 + 2 sub, +1), c < D/32,
//     of q and k (and likewise of v and o with V), so each row is read as 16
//     consecutive 4- or 8-byte words per pair of elements;
//   * the q.k dot of a thread runs the four fp32 chains of sdpa_kernel (its k-th
//     element to chain (k/2 % 2)*2 + k%2), summed (c0 + c1) + (c2 + c3), then a
//     xor-butterfly over the 16 threads -- the lane split bi_oracle.c follows with
//     lanes = 16 and two-element vectors;
//   * K and V rows stream through a ring of 32-key stages (one key per partial).
// ---------------------------------------------------------------------------
constexpr int GEN_LP = 16;
constexpr int GEN_NT = PARTIALS * GEN_LP;  // 512 threads

// Elements e and e + 1 (e even) of a row in shared memory, widened to an fp32 pair.
template <typename T>
__device__ __forceinline__ f2 load_pair(const T* row, int e) {
  if constexpr (sizeof(T) == 4) {
    const float2 w = *reinterpret_cast<const float2*>(row + e);
    return pack2(w.x, w.y);
  } else if constexpr (dtype_of<T>::value == 2) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + e);
    return f2{static_cast<uint64_t>(w << 16) | (static_cast<uint64_t>(w & 0xffff0000u) << 32)};
  } else {
    const float2 fl = __half22float2(*reinterpret_cast<const __half2*>(row + e));
    return pack2(fl.x, fl.y);
  }
}

template <typename T, int EMAX, int EVMAX>
__global__ void __launch_bounds__(GEN_NT, 1) sdpa_generic_kernel(const Params p, int stages) {
  constexpr int NW = GEN_NT / 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const int D = p.D, V = p.V;
  const int E2 = D / 32, EV2 = V / 32;  // element pairs per thread
  T* sK = reinterpret_cast<T*>(smem);
  T* sV = sK + static_cast<int64_t>(stages) * PARTIALS * D;
  uint8_t* tail = reinterpret_cast<uint8_t*>(sV + static_cast<int64_t>(stages) * PARTIALS * V);
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(tail) + 7) & ~static_cast<uintptr_t>(7));
  int* done_count = reinterpret_cast<int*>(full + stages);  // [stages]
  int* issued_count = done_count + stages;
  volatile int* abort_flag = issued_count + 1;
  float* comb_m = reinterpret_cast<float*>(done_count + stages + 4);  // [PARTIALS]
  float* comb_l = comb_m + PARTIALS;                                  // [PARTIALS + 1]
  float* comb_o = reinterpret_cast<float*>(smem);  // [PARTIALS][V], after the walk

  const int tid = threadIdx.x;
  const int part = tid / GEN_LP;
  const int sub = tid % GEN_LP;
  const int lane = tid & 31;

  int idx = blockIdx.x;
  const int s = idx % p.qL;
  idx /= p.qL;
  const int h = idx % p.H;
  const int b = idx / p.H;
  const int kvh = h / (p.H / p.Hkv);

  int64_t kmax = p.N;
  if (p.mask_mode == 1) {
    const int64_t last = p.causal_offset + s;
    kmax = last < 0 ? 0 : (last + 1 < p.N ? last + 1 : p.N);
  }
  const int nblocks = static_cast<int>((kmax + PARTIALS - 1) / PARTIALS);

  const T* Kb = static_cast<const T*>(p.k) + static_cast<int64_t>(b) * p.ks0 +
                static_cast<int64_t>(kvh) * p.ks1;
  const T* Vb = static_cast<const T*>(p.v) + static_cast<int64_t>(b) * p.vs0 +
                static_cast<int64_t>(kvh) * p.vs1;
  const T* Mk = static_cast<const T*>(p.mask);
  const T* mrow = Mk == nullptr ? nullptr
                                : Mk + static_cast<int64_t>(b) * p.ms0 +
                                      static_cast<int64_t>(h) * p.ms1 + static_cast<int64_t>(s) * p.ms2;
  const T* qrow = static_cast<const T*>(p.q) + static_cast<int64_t>(b) * p.qs0 +
                  static_cast<int64_t>(h) * p.qs1 + static_cast<int64_t>(s) * p.qs2;

  // q pre-scaled in fp32; o zero.  Pair c of the thread: elements 2 (c*16 + sub), +1.
  f2 qv[EMAX / 2], o[EVMAX / 2];
  const f2 sc = pack2(p.scale, p.scale);
#pragma unroll
  for (int c = 0; c < EMAX / 2; ++c) {
    if (c < E2) {
      const int e = 2 * (c * GEN_LP + sub);
      qv[c] = mul2(sc, pack2(to_f32(qrow[e]), to_f32(qrow[e + 1])));
    }
  }
#pragma unroll
  for (int c = 0; c < EVMAX / 2; ++c) o[c] = f2{0};
  float m = -3.40282347e+38f;
  float l = 0.f;
  const T* Sk = static_cast<const T*>(p.sinks);
  if (Sk != nullptr && part == 0) {
    m = to_f32(Sk[h]);
    l = 1.f;
  }

  const uint32_t krow_bytes = static_cast<uint32_t>(D) * sizeof(T);
  const uint32_t vrow_bytes = static_cast<uint32_t>(V) * sizeof(T);
  auto issue = [&](int blk) {
    const int st = blk % stages;
    const int64_t i0 = static_cast<int64_t>(blk) * PARTIALS;
    const int64_t rows = (kmax - i0) < PARTIALS ? (kmax - i0) : PARTIALS;
    const uint32_t kb = static_cast<uint32_t>(rows) * krow_bytes;
    const uint32_t vb = static_cast<uint32_t>(rows) * vrow_bytes;
    mbar_arrive_expect_tx(&full[st], kb + vb);
    bulk_load(sK + static_cast<int64_t>(st) * PARTIALS * D, Kb + i0 * D, kb, &full[st]);
    bulk_load(sV + static_cast<int64_t>(st) * PARTIALS * V, Vb + i0 * V, vb, &full[st]);
  };

  if (tid == 0) {
    for (int st = 0; st < stages; ++st) {
      mbar_init(&full[st], 1);
      done_count[st] = 0;
    }
    *abort_flag = 0;
    fence_barrier_init();
    int n0 = 0;
    for (; n0 < stages && n0 < nblocks; ++n0) issue(n0);
    *issued_count = n0;
  }
  __syncthreads();

  bool aborted = false;
  for (int t = 0; t < nblocks; ++t) {
    const int st = t % stages;
    bool ok = mbar_wait(&full[st], static_cast<uint32_t>((t / stages) & 1), abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) {
      if (lane == 0) {
        *abort_flag = 1;
        record_error(&g_error_word, (3u << 8) | kErrReasonTimeout);
      }
      aborted = true;
      break;
    }
    const int64_t i = static_cast<int64_t>(t) * PARTIALS + part;  // this partial's key
    const bool in_range = i < kmax;
    const T* krow = sK + (static_cast<int64_t>(st) * PARTIALS + part) * D;
    // four fp32 chains: pairs c even -> acc[0], c odd -> acc[1]
    f2 acc[2] = {f2{0}, f2{0}};
#pragma unroll
    for (int c = 0; c < EMAX / 2; ++c) {
      if (c < E2) {
        acc[c & 1] = fma2(qv[c], load_pair<T>(krow, 2 * (c * GEN_LP + sub)), acc[c & 1]);
      }
    }
    float dot = __fadd_rn(__fadd_rn(lo_of(acc[0]), hi_of(acc[0])),
                          __fadd_rn(lo_of(acc[1]), hi_of(acc[1])));
#pragma unroll
    for (int off = GEN_LP / 2; off >= 1; off >>= 1) {
      dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, off));
    }
    // scalar online-softmax step (every thread of the partial computes the same values)
    float bias = 0.f;
    bool use = in_range;
    if (p.mask_mode == 2 && in_range) {
      bias = to_f32(mrow[i]);
      use = bias > -3.0e38f;
    }
    if (use) {
      const float score = __fadd_rn(dot, bias);
      float f = 1.f, ex;
      if (score > m) {
        f = expf(__fsub_rn(m, score));
        m = score;
        ex = 1.0f;
        l = __fmaf_rn(l, f, 1.0f);
      } else {
        ex = expf(__fsub_rn(score, m));
        l = __fadd_rn(l, ex);
      }
      const T* vrow = sV + (static_cast<int64_t>(st) * PARTIALS + part) * V;
      const f2 e_2 = pack2(ex, ex);
      const f2 f_2 = pack2(f, f);
#pragma unroll
      for (int c = 0; c < EVMAX / 2; ++c) {
        if (c < EV2) {
          if (f != 1.0f) o[c] = mul2(o[c], f_2);
          o[c] = fma2(e_2, load_pair<T>(vrow, 2 * (c * GEN_LP + sub)), o[c]);
        }
      }
    }
    // The last warp to finish with this stage refills it with block t + stages.
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&done_count[st], 1) == NW - 1) {
        __threadfence_block();
        done_count[st] = 0;
        if (t + stages < nblocks && !*abort_flag) {
          fence_proxy_async_smem();
          issue(t + stages);
          atomicMax(issued_count, t + stages + 1);
        }
      }
    }
  }
  if (__syncthreads_or(aborted)) {
    if (tid == 0) {
      const int issued = *issued_count;
      for (int blk = issued - stages < 0 ? 0 : issued - stages; blk < issued; ++blk) {
        mbar_wait(&full[blk % stages], static_cast<uint32_t>((blk / stages) & 1), nullptr);
      }
    }
    return;
  }
  __syncthreads();  // every stage consumed: the ring is free for the combine

#pragma unroll
  for (int c = 0; c < EVMAX / 2; ++c) {
    if (c < EV2) {
      const int e = 2 * (c * GEN_LP + sub);
      *reinterpret_cast<float2*>(&comb_o[part * V + e]) = make_float2(lo_of(o[c]), hi_of(o[c]));
    }
  }
  if (sub == 0) {
    comb_m[part] = m;
    comb_l[part] = l;
  }
  __syncthreads();
  if (tid < 32) {
    const float ls = combine_weights(comb_m, comb_l, tid);  // comb_m now holds f_q
    if (tid == 0) comb_l[PARTIALS] = ls;
  }
  __syncthreads();
  const float lsum = comb_l[PARTIALS];
  T* O = static_cast<T*>(p.out);
  for (int j = tid; j < V; j += GEN_NT) {
    float a = 0.f;
#pragma unroll 8
    for (int q = 0; q < PARTIALS; ++q) a = __fmaf_rn(comb_o[q * V + j], comb_m[q], a);
    const float res = lsum == 0.f ? a : __fdiv_rn(a, lsum);
    O[static_cast<int64_t>(b) * p.os0 + static_cast<int64_t>(h) * p.os1 +
      static_cast<int64_t>(s) * p.os2 + j] = from_f32<T>(res);
  }
}

// Shared memory of the generic kernel at `stages` ring stages (the combine reuses the
// ring, so the ring is made at least as large as its 32 x V floats).
static int64_t generic_smem(int64_t D, int64_t V, int64_t es, int stages) {
  int64_t ring = static_cast<int64_t>(stages) * PARTIALS * (D + V) * es;
  const int64_t comb = static_cast<int64_t>(PARTIALS) * V * 4;
  if (ring < comb) ring = comb;
  return ring + 8 + static_cast<int64_t>(stages) * 8 + 4 * (stages + 4) + (2 * PARTIALS + 1) * 4;
}

template <typename T, int EMAX, int EVMAX>
static int launch_generic_t(const SdpaArgs& a, const Params& p, cudaStream_t stream) {
  const int64_t es = sizeof(T);
  const int64_t stage_bytes = PARTIALS * (a.D + a.V) * es;
  int stages = static_cast<int>((160 * 1024) / stage_bytes);
  if (stages > 4) stages = 4;
  if (stages < 2) stages = 2;
  const int64_t smem = generic_smem(a.D, a.V, es, stages);
  if (smem > 227 * 1024) {
    return set_error(BI_ERR_UNSUPPORTED, "head dims D=%lld V=%lld are too large for one CTA",
                     static_cast<long long>(a.D), static_cast<long long>(a.V));
  }
  auto kern = sdpa_generic_kernel<T, EMAX, EVMAX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(sdpa generic)");
  const int64_t blocks = a.B * a.H * a.qL;
  if (blocks > 0x7fffffffLL) return set_error(BI_ERR_UNSUPPORTED, "too many attention rows");
  kern<<<static_cast<unsigned>(blocks), GEN_NT, static_cast<size_t>(smem), stream>>>(p, stages);
  return cuda_status(cudaGetLastError(), "sdpa generic launch");
}

// Register arrays sized for the head dims: up to 256 or up to 640 elements.
template <typename T>
static int launch_generic(const SdpaArgs& a, const Params& p, cudaStream_t stream) {
  const int64_t lim = sizeof(T) == 4 ? 384 : 640;
  if (a.D > lim || a.V > lim || (sizeof(T) == 4 && a.D + a.V > 768)) {
    return set_error(BI_ERR_UNSUPPORTED,
                     "head dims D=%lld V=%lld are not built (multiples of 32; D, V <= 640 for "
                     "16-bit types; D, V <= 384 and D + V <= 768 for float32)",
                     static_cast<long long>(a.D), static_cast<long long>(a.V));
  }
  const bool wd = a.D > 256, wv = a.V > 256;
  if (!wd && !wv) return launch_generic_t<T, 16, 16>(a, p, stream);
  if (wd && !wv) return launch_generic_t<T, 40, 16>(a, p, stream);
  if (!wd && wv) return launch_generic_t<T, 16, 40>(a, p, stream);
  return launch_generic_t<T, 40, 40>(a, p, stream);
}

// ---------------------------------------------------------------------------
// Tensor-core route: fp16 / bf16, D = 64 or 128.
//
// The same fold -- key i belongs to partial i % 32, each partial keeps an fp32
// online-softmax state, the 32 partials are combined in the fixed order p = 0..31 --
// with a partial's keys folded a stage at a time.  Keys arrive in stages of 128
// (4 per partial, at absolute positions fixed by the key index alone), and each
// (query head h, partial p) takes the visible ones among its 4 at once:
//     m' = max(m, max_j s_j);  f = exp(m - m');  e_j = exp(s_j - m')
//     l  = fmaf(l, f, (e_0 + e_1) + (e_2 + e_3));  o = o * f + sum_j e_j v_j
// (f = 1 exactly when m' == m, and the multiply is skipped; a stage in which none of
// a partial's keys is visible leaves its state untouched).
//
// The products run on the tensor cores with mma.sync m16n8k16 and fp32 accumulation
// (at decode the pipe is far from busy; the kernel is bound by streaming K and V).
// MMA rows are (head, partial) pairs, r = pp*GH + h inside a warp of 16 rows, so the
// GQA group shares every K/V fragment.  A partial's 4 keys of a stage occupy
// positions 4*j + p % 4 of a 16-key MMA step, for every GQA factor; the other
// positions of the row carry exact zeros.  s = scale * (q . k) with q and k as
// given; e enters the second product as e_hi + e_lo, two 16-bit values holding ~16
// significant bits.  K and V stages come in by 4-D TMA (128-byte swizzle, zero fill
// past N), one TMA box per 64 columns.
namespace tcr {

constexpr int R = 4;                 // keys per partial per stage
constexpr int KEYS = PARTIALS * R;   // keys per stage
constexpr int BOX_D = 64;            // columns per TMA box (128-byte rows)

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (dtype_of<T>::value == 2) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Shared-memory address of the 16-byte chunk holding columns [d, d + 8) of stage row
// `row`: one TMA box per 64 columns (KEYS rows of 128 B), chunks swizzled by row % 8.
__device__ __forceinline__ uint32_t kv_addr(uint32_t base, int row, int d) {
  const int box = d >> 6;
  const int c = (d & 63) >> 3;
  return base + box * (KEYS * 128) + row * 128 + ((c ^ (row & 7)) << 4);
}

// ---------------------------------------------------------------------------------
// GQA kernel: q.k on the tensor cores, the fold and P.V on the CUDA cores.
//
// One CTA per (batch, query row, GH = 4, 2 or 1 query heads of one KV head), 256
// threads, 128-key stages.  Thread (p, sl) -- p = tid / 8 the partial, sl = tid % 8 --
// owns, for the GH heads, o[h][d] of partial p for the columns d = 64 c + 8 sl + [0, 8).
// Per stage t:
//   A. scores: warp w computes S[key][head] = k_key . q_head for keys 16w .. 16w+15
//      as one m16n8k16 MMA chain over the head dim (A = 16 K rows from shared memory,
//      B = the GH q rows -- the other columns zero), fp32 accumulation, into shared
//      memory.  Every K fragment serves all GH heads.
//   B. fold: the 8 threads of partial p hold its GH x 4 (head, key) pairs of the stage
//      (keys 32 j + p; 8 / GH threads per head: two keys each for GH = 4, one for GH =
//      2, one twice over for GH = 1) and, per head, the state (m, l) in each of them:
//          x_j = scale * S (+ mask),  m' = max(m, max_j x_j),  e_j = exp(x_j - m'),
//          f = exp(m - m'),  l = fmaf(l, f, (e_0 + e_1) + (e_2 + e_3)),
//      the max and the two pair sums crossing the head's threads by shuffle; the
//      weights reach the other threads of the partial by shuffle (-0.0 marks a key
//      that is not visible: exp never returns it).
//   C. numerator: o = o * f (skipped when f == 1), then o = fmaf(e_j, v_j, o) for the
//      visible keys j = 0..3 in order, in fp32 (packed fma.rn.f32x2): the weights
//      enter exactly.  Each V row is read once for the 4 heads.
// K and V of a stage complete on separate barriers: a K slot refills as soon as the
// stage's scores are out, while its fold and P.V still run.  A row's arithmetic depends
// on its own q row, the keys and the mask only: an MMA column is one head whatever the
// others hold, and every other step is per (head, partial).  GH and the ring depth
// decide which CTA, thread and buffer run a step, never the step.
template <int D, int GH_, int S_>
struct GqaPlan {
  static constexpr int GH = GH_;
  static constexpr int NT = 256;
  static constexpr int NCH = D / 64;        // 16-byte V vectors per thread per key
  static constexpr int TSB = KEYS * D * 2;  // one tensor's stage bytes
  static constexpr int STAGES = S_;
  static constexpr int XP = KEYS + 8;       // score row pitch (distinct banks for phase B)
  static constexpr int COMB = GH * PARTIALS * D * 4 + 2 * GH * PARTIALS * 4 + 64;
  static constexpr int REGION = 2 * STAGES * TSB > COMB ? 2 * STAGES * TSB : COMB;
  static constexpr int SMEM = 1024 + REGION + GH * XP * 4 + 2 * STAGES * 8 + 64;
  // D = 64 with one stage: three CTAs per SM fit (37 KB each, at most 85 registers a
  // thread without spills); measured 7-11 % faster on prefill, equal on decode
  static constexpr int CTAS_PER_SM =
      (D == 64 && S_ == 1) ? 3 : (2 * SMEM <= 227 * 1024 ? 2 : 1);
  static_assert(SMEM <= 227 * 1024, "the stage ring must fit");
  static_assert(CTAS_PER_SM * SMEM <= 227 * 1024, "the CTAs of an SM must fit");
};

// 8 consecutive 16-bit values -> 4 fp32 pairs (exact).
template <typename T>
__device__ __forceinline__ void widen8(const uint4 x, f2 (&v)[4]) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (dtype_of<T>::value == 2) {
      v[i] = pack2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[i] = pack2(f.x, f.y);
    }
  }
}

constexpr uint32_t kHiddenKey = 0x80000000u;  // -0.0f: the weight of a key not visible

template <typename T, int D, int GH_, int S>
__global__ void __launch_bounds__(256, (GqaPlan<D, GH_, S>::CTAS_PER_SM))
    sdpa_gqa_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const Params p) {
  using PL = GqaPlan<D, GH_, S>;
  constexpr int GH = PL::GH;
  constexpr int NT = PL::NT;
  constexpr int NCH = PL::NCH;
  constexpr int KSTEPS = D / 16;  // MMA k-steps over the head dim
  constexpr int STAGES = PL::STAGES;
  constexpr int TSB = PL::TSB;
  constexpr int XP = PL::XP;
  static_assert(NT / 32 * 16 == KEYS, "one 16-key MMA tile per warp");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + STAGES * TSB;
  float* xs = reinterpret_cast<float*>(smem + PL::REGION);  // scores [GH][XP]
  // K and V of a stage complete on their own barriers, so a K slot refills as soon as
  // its scores are out, while the fold and P.V of the stage still run
  uint64_t* full_k = reinterpret_cast<uint64_t*>(xs + GH * XP);
  uint64_t* full_v = full_k + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full_v + STAGES);
  int* issued_k = const_cast<int*>(abort_flag) + 1;
  int* issued_v = issued_k + 1;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int gq = lane >> 2;
  const int q4 = lane & 3;

  const int groups = p.H / GH;
  int idx = blockIdx.x;
  const int s = idx % p.qL;
  idx /= p.qL;
  const int hg = idx % groups;
  const int b = idx / groups;
  const int h0 = hg * GH;
  const int kvh = h0 / (p.H / p.Hkv);

  int64_t kmax = p.N;
  if (p.mask_mode == 1) {
    const int64_t last = p.causal_offset + s;
    kmax = last < 0 ? 0 : (last + 1 < p.N ? last + 1 : p.N);
  }
  const int nblocks = static_cast<int>((kmax + KEYS - 1) / KEYS);

  // Phase A operand: q of head gq (columns 4..7 of B are zero).
  uint32_t qb[KSTEPS][2];
  {
    const T* Q = static_cast<const T*>(p.q) + static_cast<int64_t>(b) * p.qs0 +
                 static_cast<int64_t>(h0 + (gq < GH ? gq : 0)) * p.qs1 +
                 static_cast<int64_t>(s) * p.qs2;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      qb[kk][0] = gq < GH ? *reinterpret_cast<const uint32_t*>(Q + 16 * kk + 2 * q4) : 0u;
      qb[kk][1] = gq < GH ? *reinterpret_cast<const uint32_t*>(Q + 16 * kk + 8 + 2 * q4) : 0u;
    }
  }
  // Phases B and C: partial cp; in B head bh, keys of index wi among the head's TPH.
  constexpr int TPH = 8 / GH;           // threads per head in a partial's 8
  constexpr int KPT = GH == 4 ? 2 : 1;  // keys per thread in B
  const int cp = tid >> 3;
  const int sl = tid & 7;
  const int bh = sl / TPH;
  const int wi = sl % TPH;
  const int grp = lane & ~7;  // first lane of this partial's 8
  float m = -3.40282347e+38f, l = 0.f;  // state of (head bh, partial cp), in each of its threads
  {
    const T* Sk = static_cast<const T*>(p.sinks);
    if (Sk != nullptr && cp == 0) {
      m = to_f32(Sk[h0 + bh]);
      l = 1.f;
    }
  }
  const T* mrow = p.mask_mode == 2
                      ? static_cast<const T*>(p.mask) + static_cast<int64_t>(b) * p.ms0 +
                            static_cast<int64_t>(h0 + bh) * p.ms1 + static_cast<int64_t>(s) * p.ms2
                      : nullptr;
  f2 o[GH][NCH][4];
#pragma unroll
  for (int h = 0; h < GH; ++h)
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[h][c][i] = pack2(0.f, 0.f);

  // one tensor's 128-key block into its ring slot (tid 0 only)
  auto issue = [&](const CUtensorMap* map, uint8_t* ring, uint64_t* bars, int* issued, int blk) {
    const int st = blk % STAGES;
    mbar_arrive_expect_tx(&bars[st], TSB);
#pragma unroll
    for (int bx = 0; bx < D / BOX_D; ++bx) {
      tma_load_4d(ring + st * TSB + bx * KEYS * 128, map, &bars[st], bx * BOX_D, blk * KEYS, kvh, b);
    }
    *issued = blk + 1;
  };
  // A: scores of stage block t (its K in ring slot t % STAGES) into buffer xb.
  auto scores = [&](int t, float* xb) {
    const uint32_t kbase = smem_u32(sK + (t % STAGES) * TSB);
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    const int mi = lane >> 3;
    const int krow = 16 * warp + (lane & 7) + 8 * (mi & 1);
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, kv_addr(kbase, krow, 16 * kk + 8 * (mi >> 1)));
      mma16816<T>(c, a[0], a[1], a[2], a[3], qb[kk][0], qb[kk][1]);
    }
    // columns 2 q4, 2 q4 + 1 are heads (those below GH); rows gq and gq + 8 keys
    const int k0 = 16 * warp + gq;
    if (2 * q4 < GH) {
      xb[(2 * q4) * XP + k0] = c[0];
      xb[(2 * q4) * XP + k0 + 8] = c[2];
    }
    if (2 * q4 + 1 < GH) {
      xb[(2 * q4 + 1) * XP + k0] = c[1];
      xb[(2 * q4 + 1) * XP + k0 + 8] = c[3];
    }
  };
  // Every thread waits; the result is made warp-uniform, since the MMAs, ldmatrix and
  // shuffles that follow need the whole warp.
  auto wait_on = [&](uint64_t* bars, int t) {
    const bool w = mbar_wait(&bars[t % STAGES], static_cast<uint32_t>((t / STAGES) & 1), abort_flag);
    return __all_sync(0xffffffffu, w) != 0;
  };

  if (tid == 0) {
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&full_k[st], 1);
      mbar_init(&full_v[st], 1);
    }
    *abort_flag = 0;
    *issued_k = 0;
    *issued_v = 0;
    fence_barrier_init();
    for (int n0 = 0; n0 < STAGES && n0 < nblocks; ++n0) {
      issue(&tk, sK, full_k, issued_k, n0);
      issue(&tv, sV, full_v, issued_v, n0);
    }
  }
  __syncthreads();

  const float scale = p.scale;
  bool aborted = false;
  for (int t = 0; t < nblocks; ++t) {
    const int st = t % STAGES;
    float* xb = xs;
    const bool ok = wait_on(full_k, t);
    if (ok) scores(t, xb);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        *abort_flag = 1;
        record_error(&g_error_word, (2u << 8) | kErrReasonTimeout);
      }
      aborted = true;
      break;
    }
    // every warp is done with this block's A: its K slot is free
    if (tid == 0 && t + STAGES < nblocks) {
      fence_proxy_async_smem();
      issue(&tk, sK, full_k, issued_k, t + STAGES);
    }
    const int64_t key0 = static_cast<int64_t>(t) * KEYS;

    // ---- B: head bh, keys j(u) of partial cp
    float x[KPT];
    bool use[KPT];
#pragma unroll
    for (int u = 0; u < KPT; ++u) {
      const int j = GH == 4 ? 2 * wi + u : (wi & 3);
      const int64_t key = key0 + 32 * j + cp;
      bool vis = key < kmax;
      float v = __fmul_rn(xb[bh * XP + 32 * j + cp], scale);
      if (vis && mrow != nullptr) {
        const float bias = to_f32(mrow[key]);
        vis = bias > -3.0e38f;
        v = __fadd_rn(v, bias);
      }
      use[u] = vis;
      x[u] = v;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int u = 0; u < KPT; ++u)
      if (use[u]) mx = fmaxf(mx, x[u]);
    // the head's 4 keys sit in lanes differing in bit 0 (GH = 4) or bits 0-1
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    if (GH < 4) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const bool any = mx != -INFINITY;
    const float mn = any ? fmaxf(m, mx) : m;
    float ev[KPT];
#pragma unroll
    for (int u = 0; u < KPT; ++u) ev[u] = use[u] ? expf(__fsub_rn(x[u], mn)) : __uint_as_float(kHiddenKey);
    const float e0 = ev[0];
    const float e1 = ev[KPT - 1];
    // (e_0 + e_1) + (e_2 + e_3); IEEE addition is commutative, so every thread of the
    // head gets the same sum whichever half it holds
    float pair;
    if (GH == 4) {
      pair = __fadd_rn(use[0] ? e0 : 0.f, use[KPT - 1] ? e1 : 0.f);
    } else {
      const float mine = use[0] ? e0 : 0.f;
      pair = __fadd_rn(mine, __shfl_xor_sync(0xffffffffu, mine, 1));
    }
    const float pair_other = __shfl_xor_sync(0xffffffffu, pair, GH == 4 ? 1 : 2);
    float f = 1.0f;
    if (any) {
      const float sum = __fadd_rn(pair, pair_other);
      f = mn == m ? 1.0f : expf(__fsub_rn(m, mn));
      l = __fmaf_rn(l, f, sum);
      m = mn;
    }

    // ---- C: o = o * f, then o = fmaf(e_j, v_j, o) for the visible keys, j ascending
    const bool ok_v = wait_on(full_v, t);
    const uint32_t vbase = smem_u32(sV + st * TSB);
    if (ok_v) {
#pragma unroll
    for (int h = 0; h < GH; ++h) {
      const float fh = __shfl_sync(0xffffffffu, f, grp + TPH * h);
      if (fh != 1.0f) {
        const f2 ff = pack2(fh, fh);
#pragma unroll
        for (int c2 = 0; c2 < NCH; ++c2)
#pragma unroll
          for (int i = 0; i < 4; ++i) o[h][c2][i] = mul2(o[h][c2][i], ff);
      }
    }
#pragma unroll
    for (int j = 0; j < R; ++j) {
      f2 v[NCH][4];
#pragma unroll
      for (int c2 = 0; c2 < NCH; ++c2) {
        uint4 raw;
        asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(raw.x), "=r"(raw.y), "=r"(raw.z), "=r"(raw.w)
                     : "r"(kv_addr(vbase, 32 * j + cp, 64 * c2 + 8 * sl)));
        widen8<T>(raw, v[c2]);
      }
      // weight of (head h, key j): GH = 4: thread 2 h + j / 2 of the partial, its
      // e_{j % 2}; else thread TPH h + j
      const float mine = (GH == 4 && (j & 1)) ? e1 : e0;
#pragma unroll
      for (int h = 0; h < GH; ++h) {
        const float eh =
            __shfl_sync(0xffffffffu, mine, grp + TPH * h + (GH == 4 ? (j >> 1) : j));
        if (__float_as_uint(eh) != kHiddenKey) {
          const f2 ee = pack2(eh, eh);
#pragma unroll
          for (int c2 = 0; c2 < NCH; ++c2)
#pragma unroll
            for (int i = 0; i < 4; ++i) o[h][c2][i] = fma2(ee, v[c2][i], o[h][c2][i]);
        }
      }
    }
    }  // ok_v

    if (__syncthreads_or(!ok_v)) {  // stage st's V and the scores are free
      if (tid == 0) {
        *abort_flag = 1;
        record_error(&g_error_word, (2u << 8) | kErrReasonTimeout);
      }
      aborted = true;
      break;
    }
    if (tid == 0 && t + STAGES < nblocks) {
      fence_proxy_async_smem();
      issue(&tv, sV, full_v, issued_v, t + STAGES);
    }
  }
  if (aborted) {
    if (tid == 0) {
      // wait, bounded, for every copy still in flight before the CTA leaves
      const int ik = *issued_k, iv = *issued_v;
      for (int blk = ik - STAGES < 0 ? 0 : ik - STAGES; blk < ik; ++blk) {
        mbar_wait(&full_k[blk % STAGES], static_cast<uint32_t>((blk / STAGES) & 1), nullptr);
      }
      for (int blk = iv - STAGES < 0 ? 0 : iv - STAGES; blk < iv; ++blk) {
        mbar_wait(&full_v[blk % STAGES], static_cast<uint32_t>((blk / STAGES) & 1), nullptr);
      }
    }
    return;
  }
  __syncthreads();  // every stage consumed and no copy in flight: the ring is free

  // ---- combine the 32 partials of every head, p = 0..31 (as the CUDA-core route)
  float* comb_o = reinterpret_cast<float*>(smem);  // [GH][32][D]
  float* comb_m = comb_o + GH * PARTIALS * D;      // [GH][32]
  float* comb_l = comb_m + GH * PARTIALS;          // [GH][32]
  float* comb_s = comb_l + GH * PARTIALS;          // [GH] denominators
#pragma unroll
  for (int h = 0; h < GH; ++h) {
#pragma unroll
    for (int c2 = 0; c2 < NCH; ++c2) {
      float4* dst = reinterpret_cast<float4*>(comb_o + (h * PARTIALS + cp) * D + 64 * c2 + 8 * sl);
      dst[0] = make_float4(lo_of(o[h][c2][0]), hi_of(o[h][c2][0]), lo_of(o[h][c2][1]),
                           hi_of(o[h][c2][1]));
      dst[1] = make_float4(lo_of(o[h][c2][2]), hi_of(o[h][c2][2]), lo_of(o[h][c2][3]),
                           hi_of(o[h][c2][3]));
    }
  }
  if (wi == 0) {
    comb_m[bh * PARTIALS + cp] = m;
    comb_l[bh * PARTIALS + cp] = l;
  }
  __syncthreads();
  if (warp < GH) {
    const float ls = combine_weights(comb_m + warp * PARTIALS, comb_l + warp * PARTIALS, lane);
    if (lane == 0) comb_s[warp] = ls;  // comb_m now holds the f_q of each head
  }
  __syncthreads();
  T* O = static_cast<T*>(p.out);
  for (int jj = tid; jj < GH * D; jj += NT) {
    const int hh = jj / D;
    const int j = jj - hh * D;
    const float* fq = comb_m + hh * PARTIALS;
    const float lsum = comb_s[hh];
    float acc = 0.f;
#pragma unroll 8
    for (int q = 0; q < PARTIALS; ++q) acc = __fmaf_rn(comb_o[(hh * PARTIALS + q) * D + j], fq[q], acc);
    const float res = lsum == 0.f ? acc : __fdiv_rn(acc, lsum);
    O[static_cast<int64_t>(b) * p.os0 + static_cast<int64_t>(h0 + hh) * p.os1 +
      static_cast<int64_t>(s) * p.os2 + j] = from_f32<T>(res);
  }
}

}  // namespace tcr

// Threads per partial: 32 bytes of a key row per thread where the row allows, a power
// of two that divides D, at most 16 (CTAs of at most 512 threads).  A function of
// (D, dtype) only.
template <typename T>
constexpr int lanes_for(int D) {
  int lp = (D * static_cast<int>(sizeof(T))) / 32;
  if (lp > 16) lp = 16;
  if (lp < 1) lp = 1;
  int p2 = 1;
  while (p2 * 2 <= lp) p2 *= 2;
  while (p2 > 1 && D % p2 != 0) p2 /= 2;
  return p2;
}

// Shared-memory plan per (dtype, D): ROWS key rows per partial per stage and STAGES
// stages, within ~96 KB of K/V ring (at least 2 stages, at most 4).
template <typename T, int D>
constexpr int rows_for() {
  constexpr int row_pair = 2 * PARTIALS * D * static_cast<int>(sizeof(T));  // K+V, 1 row
  return (BI_SDPA_ROWS_PER_STAGE * row_pair * 2 <= 128 * 1024) ? BI_SDPA_ROWS_PER_STAGE : 1;
}

template <typename T, int D>
constexpr int stages_for() {
  constexpr int pair = 2 * PARTIALS * rows_for<T, D>() * D * static_cast<int>(sizeof(T));
  constexpr int s = (96 * 1024) / pair;
  return s < 2 ? 2 : (s > 4 ? 4 : s);
}

// Largest heads-per-CTA the register budget allows: HG * 2E fp32 values of q and o
// per thread within BI_SDPA_REG_BUDGET.
template <typename T, int D>
constexpr int max_heads_per_cta() {
  constexpr int LP = lanes_for<T>(D);
  constexpr int E = D / LP;
  constexpr int budget = BI_SDPA_REG_BUDGET;
  return (8 * E <= budget) ? 4 : (4 * E <= budget) ? 2 : 1;
}

template <typename T, int D, int HG>
static int launch_hg(const Params& p, int64_t blocks, cudaStream_t stream) {
  constexpr int LP = lanes_for<T>(D);
  constexpr int S = stages_for<T, D>();
  constexpr int R = rows_for<T, D>();
  constexpr int NT = PARTIALS * LP;
  constexpr int smem = 2 * S * PARTIALS * R * D * static_cast<int>(sizeof(T)) + S * 8 +
                       4 * (S + 4) + (2 * PARTIALS + 1) * 4;
  static_assert(PARTIALS * D * 4 <= 2 * S * PARTIALS * R * D * static_cast<int>(sizeof(T)),
                "combine buffer must fit in the stage ring");
  static_assert(smem <= 227 * 1024, "shared memory above the per-CTA limit");
  auto kern = sdpa_kernel<T, D, LP, HG, S, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(sdpa)");
  // Ask for the largest shared-memory carveout so two CTAs' stage rings fit per SM.
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(sdpa carveout)");
  if (blocks > 0x7fffffffLL) return set_error(BI_ERR_UNSUPPORTED, "too many attention rows");
  kern<<<static_cast<unsigned>(blocks), NT, smem, stream>>>(p);
  return cuda_status(cudaGetLastError(), "sdpa launch");
}

#ifndef BI_SDPA_MAX_HG
#define BI_SDPA_MAX_HG 4
#endif

template <typename T, int D>
static int launch_d(const SdpaArgs& a, const Params& p, cudaStream_t stream) {
  constexpr int HGMAX = max_heads_per_cta<T, D>() < BI_SDPA_MAX_HG ? max_heads_per_cta<T, D>()
                                                                  : BI_SDPA_MAX_HG;
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

namespace tcr {

// K or V as a 4-D TMA map (D, N, Hkv, B): rows of a head are contiguous; a dimension
// of extent 1 gets a compact stride, any other must be a positive multiple of 16 B.
template <int D>
static int kv_map(CUtensorMap* map, const void* base, const int64_t (&st)[2], const SdpaArgs& a) {
  const uint64_t rows = a.N > 0 ? static_cast<uint64_t>(a.N) : 1;
  uint64_t dims[4] = {static_cast<uint64_t>(D), rows, static_cast<uint64_t>(a.Hkv),
                      static_cast<uint64_t>(a.B)};
  uint64_t strides[3] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(st[1]) * 2,
                         static_cast<uint64_t>(st[0]) * 2};
  if (dims[2] == 1) strides[1] = strides[0] * dims[1];
  if (dims[3] == 1) strides[2] = strides[1] * dims[2];
  for (int i = 1; i < 3; ++i) {
    if (strides[i] == 0 || strides[i] % 16 != 0) {
      return set_error(BI_ERR_MISALIGNED, "k/v head and batch strides must be positive "
                                          "multiples of 8 elements");
    }
  }
  uint32_t box[4] = {BOX_D, KEYS, 1, 1};
  return encode_tiled16(map, base, 4, dims, strides, box, a.dtype);
}

template <typename T, int D, int GH, int S>
static int launch_gqa(const SdpaArgs& a, const Params& p, cudaStream_t stream) {
  using PL = GqaPlan<D, GH, S>;
  CUtensorMap tk, tv;
  int st = kv_map<D>(&tk, a.k, a.ks, a);
  if (st) return st;
  st = kv_map<D>(&tv, a.v, a.vs, a);
  if (st) return st;
  auto kern = sdpa_gqa_kernel<T, D, GH, S>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       PL::SMEM);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(sdpa gqa)");
  const int64_t blocks = a.B * (a.H / PL::GH) * a.qL;
  if (blocks > 0x7fffffffLL) return set_error(BI_ERR_UNSUPPORTED, "too many attention rows");
  kern<<<static_cast<unsigned>(blocks), PL::NT, PL::SMEM, stream>>>(tk, tv, p);
  return cuda_status(cudaGetLastError(), "sdpa gqa launch");
}

// Heads per CTA and ring depth: GH = 4 shares each K/V stage between four heads; a grid
// with few CTAs takes GH = 2 or 1 (the next GH while twice the CTAs still fit on the
// SMs), which puts more SMs on the same keys (a KV head's stages then arrive once per
// CTA, mostly from L2).  A grid with more CTAs than SMs runs two 1-stage CTAs per SM
// (each covers the other's load latency), a smaller one a 3-stage ring per SM.
// Measured on B200 (decode, L = 8192): GH = 2 with two 1-stage CTAs per SM for a
// 512-row grid ran 160 us against 139 us for GH = 4 with one 3-stage CTA per SM; at
// D = 64 this plan beat two 3-stage CTAs per SM (235 vs 234-249 us at B = 64, H = 32;
// 71 vs 82-86 us at H = 4), and overlapping the next stage's scores with P.V gained
// nothing once K and V had separate barriers.  None of these changes a row's bits.
template <typename T, int D, int GH>
static int launch_gh(const SdpaArgs& a, const Params& p, cudaStream_t stream, bool big) {
  if (big) return launch_gqa<T, D, GH, 1>(a, p, stream);
  return launch_gqa<T, D, GH, 3>(a, p, stream);
}

template <typename T, int D>
static int launch(const SdpaArgs& a, const Params& p, cudaStream_t stream) {
  const int64_t sms = device_sm_count();
  const int64_t rows = a.B * a.H * a.qL;  // query (row, head) pairs
  int gh = 4;
  bool big;
  if (rows / 4 > sms) {
    big = true;  // two 1-stage CTAs per SM
  } else {
    while (gh > 1 && 2 * (rows / gh) <= sms) gh /= 2;
    big = false;  // one 3-stage CTA per SM
  }
  if (gh == 4) return launch_gh<T, D, 4>(a, p, stream, big);
  if (gh == 2) return launch_gh<T, D, 2>(a, p, stream, big);
  return launch_gh<T, D, 1>(a, p, stream, big);
}

}  // namespace tcr

// Route: fp16 / bf16 with D = 64 or 128 and every KV head shared by a multiple of 4
// query heads take the GQA kernel (its q.k MMAs serve the 4 heads from each K
// fragment, its fold and P.V read each V row once for them); everything else the
// CUDA-core one.  The route is a
// function of the model's shapes (dtype, D, H / Hkv) only -- never of B, qL or N -- so
// a token's bits are the same in decode and in any chunked prefill.
template <typename T>
static int launch_t(const SdpaArgs& a, const Params& p, cudaStream_t stream) {
  if (a.D != a.V || a.D > 256) return launch_generic<T>(a, p, stream);
  if constexpr (sizeof(T) == 2) {
    if ((a.H / a.Hkv) % 4 == 0) {
      if (a.D == 64) return tcr::launch<T, 64>(a, p, stream);
      if (a.D == 128) return tcr::launch<T, 128>(a, p, stream);
    }
  }
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
  p.D = static_cast<int>(a.D);
  p.V = static_cast<int>(a.V);
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
