/*
 * bi_oracle.c -- CPU restatement of mlx-batch-invariant 0.2.0's invariant GEMM and
 * attention, used as the parity checker of libbi.so.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference leg load this library; the product path never
 * does.
 *
 * Parity unpinned at the bit level: the reference's kernels are Metal source strings
 * run by MLX on Apple GPUs; neither MLX nor Metal exists on Linux, so no reference
 * output can be produced here, and the reference ships no golden vectors.  What pins
 * this restatement is (1) the reference's own test assertions -- accuracy against
 * float64, single-rounding addmm, invariance -- checked against NumPy float64 in
 * tests/test_oracle.py, and (2) the committed golden fixtures in tests/golden/.
 *
 * GEMM (mlx_batch_invariant/_gemm.py:29-130): per output element one fp32
 * accumulator, zero-initialised (:51-58), out-of-range rows and columns
 * loaded as zero (:63-80).  K is walked in slices of 8, ascending --
 * the k0-then-kk order of 8-deep MMA steps at :62-104 -- and each slice is summed in
 * order into a fresh fp32 partial, p = fmaf(a[m,k], b[k,n], p), which is then added
 * to the accumulator, acc = acc + p (Apple does not specify the order inside its
 * 8x8x8 fragment; sequential is taken).  Then the epilogue of :118-129,
 * v = alpha*acc + beta*bias with each operation rounded to fp32 (no contraction),
 * rounded once to the output type, round-to-nearest-even.
 *
 * Attention (mlx_batch_invariant/_attention.py:32-149, _mask_args :173-202): q is
 * pre-scaled in fp32 (:68-71); 32 partial online-softmax states, key i folding into
 * partial i % 32 (:89); the running max starts at the lowest finite float (:78);
 * a sink seeds partial 0 with (max = sink, sum = 1) (:80-86); causal visibility
 * i <= offset + s (:93, offset = N - qL for the reference), additive-mask keys with
 * value <= -3e38 skipped (:95-96); dot then bias (:103-106), online update (:108-115);
 * combine with the max over partials, rescale and sum (:125-141); zero output when
 * the denominator is zero (:139).  The reference sums a score with simd_sum over 32
 * lanes in an order Apple does not specify; this restatement splits the head dim
 * over `lanes` threads (each taking interleaved vectors of the row; inside a lane
 * four fmaf chains summed (c0+c1)+(c2+c3); then an xor-butterfly across lanes) --
 * the order libbi.so uses --
 * and states the update formulas as libbi.so does:
 *   m' = max(m, s); f = exp(m - m'); e = exp(s - m'); l = fmaf(l, f, e);
 *   o = fmaf(e, v, o * f); combine: l = sum fmaf(l_p, f_p, .), o = sum fmaf(o_p, f_p, .)
 * exp is the C library's expf, so results match the GPU within a few fp32 ulp, not
 * bit for bit.
 *
 * Build: oracle/build.py (gcc -O2 -ffp-contract=off -mfma -mf16c -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2 };

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float load_elem(const void* p, int64_t i, int dt) {
  switch (dt) {
    case OR_F32: return ((const float*)p)[i];
    case OR_F16: return (float)((const _Float16*)p)[i];
    default: return bf16_to_f32(((const uint16_t*)p)[i]);
  }
}

static inline void store_elem(void* p, int64_t i, float v, int dt) {
  switch (dt) {
    case OR_F32: ((float*)p)[i] = v; break;
    case OR_F16: ((_Float16*)p)[i] = (_Float16)v; break;
    default: ((uint16_t*)p)[i] = f32_to_bf16(v); break;
  }
}

/* Rounds an fp32 value to dtype and back (used by the host emulation helpers). */
float oracle_round(float v, int dt) {
  float out;
  switch (dt) {
    case OR_F32: return v;
    case OR_F16: return (float)(_Float16)v;
    default: out = bf16_to_f32(f32_to_bf16(v)); return out;
  }
}

/*
 * out[m,n] = round( alpha*acc + beta*bias[n] ) or round(acc) without bias, where
 * acc = fmaf-accumulated sum over k ascending.  b is (N,K) when b_is_nk, else (K,N).
 * Columns are processed in blocks; threads split the blocks (nthreads <= 0: all).
 */
void oracle_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, const void* bias,
                 void* out, int64_t ldo, int64_t M, int64_t N, int64_t K, int b_is_nk,
                 float alpha, float beta, int dt, int nthreads) {
  const int64_t NB = 256;
  const int64_t nblk = (N + NB - 1) / NB;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
  {
    float* bt = (float*)malloc(sizeof(float) * (size_t)(K > 0 ? K : 1) * NB);
    float* acc = (float*)malloc(sizeof(float) * NB);
    float* part = (float*)malloc(sizeof(float) * NB);
    float* arow = (float*)malloc(sizeof(float) * (size_t)(K > 0 ? K : 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (int64_t blk = 0; blk < nblk; ++blk) {
      const int64_t n0 = blk * NB;
      const int64_t nb = (N - n0) < NB ? (N - n0) : NB;
      /* B block as float, (K, nb) row-major */
      for (int64_t k = 0; k < K; ++k) {
        for (int64_t j = 0; j < nb; ++j) {
          const int64_t n = n0 + j;
          bt[k * NB + j] = b_is_nk ? load_elem(b, n * ldb + k, dt) : load_elem(b, k * ldb + n, dt);
        }
      }
      for (int64_t m = 0; m < M; ++m) {
        for (int64_t k = 0; k < K; ++k) arow[k] = load_elem(a, m * lda + k, dt);
        for (int64_t j = 0; j < nb; ++j) acc[j] = 0.0f;
        for (int64_t k0 = 0; k0 < K; k0 += 8) {
          for (int64_t j = 0; j < nb; ++j) part[j] = 0.0f;
          for (int64_t k = k0; k < k0 + 8; ++k) {
            if (k < K) {
              const float av = arow[k];
              const float* brow = bt + k * NB;
              for (int64_t j = 0; j < nb; ++j) part[j] = fmaf(av, brow[j], part[j]);
            } else {
              /* a ragged last slice is padded with zero products, as on the GPU */
              for (int64_t j = 0; j < nb; ++j) part[j] = fmaf(0.0f, 0.0f, part[j]);
            }
          }
          for (int64_t j = 0; j < nb; ++j) acc[j] = acc[j] + part[j];
        }
        for (int64_t j = 0; j < nb; ++j) {
          float v = acc[j];
          if (bias) {
            const float t1 = alpha * acc[j];
            const float t2 = beta * load_elem(bias, n0 + j, dt);
            v = t1 + t2;
          }
          store_elem(out, m * ldo + n0 + j, v, dt);
        }
      }
    }
    free(bt);
    free(acc);
    free(part);
    free(arow);
  }
}

#define PARTIALS 32

/*
 * Strides are in elements for (b, h, s) of q/out/mask and (b, h) of k/v; the last
 * dimension of every tensor is contiguous and each head block of k and v is
 * row-contiguous.  lanes: threads a key row is split over (a power of two dividing
 * D, leaving an even count per lane); here D == V (oracle_sdpa_ex takes V apart).
 */
void oracle_sdpa_ex(const void* q, const int64_t* qs, const void* k, const int64_t* ks,
                    const void* v, const int64_t* vs, const void* mask, const int64_t* ms,
                    int mask_mode, int64_t causal_offset, const void* sinks, float scale,
                    int64_t B, int64_t H, int64_t Hkv, int64_t qL, int64_t N, int64_t D,
                    int64_t V, int dt, void* out, const int64_t* os, int out_dt, int lanes,
                    int per_elems, int nthreads);

void oracle_sdpa(const void* q, const int64_t* qs, const void* k, const int64_t* ks,
                 const void* v, const int64_t* vs, const void* mask, const int64_t* ms,
                 int mask_mode, int64_t causal_offset, const void* sinks, float scale, int64_t B,
                 int64_t H, int64_t Hkv, int64_t qL, int64_t N, int64_t D, int dt, void* out,
                 const int64_t* os, int lanes, int nthreads) {
  oracle_sdpa_ex(q, qs, k, ks, v, vs, mask, ms, mask_mode, causal_offset, sinks, scale, B, H,
                 Hkv, qL, N, D, D, dt, out, os, dt, lanes, 0, nthreads);
}

/* As oracle_sdpa, with v and the output V wide (V may differ from D), the output
 * written as out_dt (OR_F32 keeps the fold's fp32 result before the final rounding to
 * the input type, for elementwise error bars), and per_elems > 0 fixing the elements
 * per vector of a lane's share of a q / k row (0: the widest of 16, 8 or 4 bytes that
 * divides the share, as libbi.so's kernels for D == V <= 256 take it; libbi.so's
 * kernel for other head dims uses 16 lanes and 2-element vectors). */
void oracle_sdpa_ex(const void* q, const int64_t* qs, const void* k, const int64_t* ks,
                    const void* v, const int64_t* vs, const void* mask, const int64_t* ms,
                    int mask_mode, int64_t causal_offset, const void* sinks, float scale,
                    int64_t B, int64_t H, int64_t Hkv, int64_t qL, int64_t N, int64_t D,
                    int64_t V, int dt, void* out, const int64_t* os, int out_dt, int lanes,
                    int per_elems, int nthreads) {
  const int64_t G = H / Hkv;
  const int64_t E = D / lanes;
  /* a lane's share of a row: vectors of W bytes (16, 8 or 4, whichever divides its
     E elements' bytes), the lanes' vectors interleaved: vector c of lane t starts at
     element (c*lanes + t)*per */
  const int64_t es = dt == OR_F32 ? 4 : 2;
  const int64_t vbytes = (E * es) % 16 == 0 ? 16 : ((E * es) % 8 == 0 ? 8 : 4);
  const int64_t per = per_elems > 0 ? per_elems : vbytes / es;
  const int64_t rows = B * H * qL;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
  {
    float* qv = (float*)malloc(sizeof(float) * D);
    float* kf = (float*)malloc(sizeof(float) * D);
    float* vf = (float*)malloc(sizeof(float) * V);
    float* o = (float*)malloc(sizeof(float) * PARTIALS * V);
    float* part = (float*)malloc(sizeof(float) * lanes);
    float* tmp = (float*)malloc(sizeof(float) * lanes);
    float m[PARTIALS], l[PARTIALS];
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
    for (int64_t r = 0; r < rows; ++r) {
      const int64_t s = r % qL;
      const int64_t h = (r / qL) % H;
      const int64_t b = r / (qL * H);
      const int64_t kvh = h / G;
      for (int64_t j = 0; j < D; ++j) qv[j] = scale * load_elem(q, b * qs[0] + h * qs[1] + s * qs[2] + j, dt);
      for (int p = 0; p < PARTIALS; ++p) {
        m[p] = -3.40282347e+38f;
        l[p] = 0.0f;
        for (int64_t j = 0; j < V; ++j) o[p * V + j] = 0.0f;
      }
      if (sinks) {
        m[0] = load_elem(sinks, h, dt);
        l[0] = 1.0f;
      }
      int64_t kmax = N;
      if (mask_mode == 1) {
        const int64_t last = causal_offset + s;
        kmax = last < 0 ? 0 : (last + 1 < N ? last + 1 : N);
      }
      const int64_t kb = b * ks[0] + kvh * ks[1];
      const int64_t vb = b * vs[0] + kvh * vs[1];
      for (int64_t i = 0; i < kmax; ++i) {
        const int p = (int)(i % PARTIALS);
        float bias = 0.0f;
        int use = 1;
        if (mask_mode == 2) {
          bias = load_elem(mask, b * ms[0] + h * ms[1] + s * ms[2] + i, dt);
          use = bias > -3.0e38f;
        }
        if (!use) continue;
        for (int64_t j = 0; j < D; ++j) kf[j] = load_elem(k, kb + i * D + j, dt);
        for (int64_t j = 0; j < V; ++j) vf[j] = load_elem(v, vb + i * V + j, dt);
        for (int t = 0; t < lanes; ++t) {
          /* four chains -- the lane's e-th element (row element ((e/per)*lanes + t)*per
             + e%per) goes to chain (e/2 % 2)*2 + e%2 -- summed (c0+c1)+(c2+c3) */
          float ch[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (int64_t e = 0; e < E; ++e) {
            const int64_t j = ((e / per) * lanes + t) * per + e % per;
            const int c = (int)(((e / 2) % 2) * 2 + e % 2);
            ch[c] = fmaf(qv[j], kf[j], ch[c]);
          }
          part[t] = (ch[0] + ch[1]) + (ch[2] + ch[3]);
        }
        for (int off = lanes / 2; off >= 1; off /= 2) {
          for (int t = 0; t < lanes; ++t) tmp[t] = part[t] + part[t ^ off];
          memcpy(part, tmp, sizeof(float) * lanes);
        }
        const float score = part[0] + bias;
        const float mnew = fmaxf(m[p], score);
        const float f = expf(m[p] - mnew);
        const float ex = expf(score - mnew);
        l[p] = fmaf(l[p], f, ex);
        for (int64_t j = 0; j < V; ++j) {
          const float scaled = o[p * V + j] * f;
          o[p * V + j] = fmaf(ex, vf[j], scaled);
        }
        m[p] = mnew;
      }
      float mx = m[0];
      for (int p = 1; p < PARTIALS; ++p) mx = fmaxf(mx, m[p]);
      float fp[PARTIALS];
      float lsum = 0.0f;
      for (int p = 0; p < PARTIALS; ++p) {
        fp[p] = expf(m[p] - mx);
        lsum = fmaf(l[p], fp[p], lsum);
      }
      for (int64_t j = 0; j < V; ++j) {
        float acc = 0.0f;
        for (int p = 0; p < PARTIALS; ++p) acc = fmaf(o[p * V + j], fp[p], acc);
        const float res = lsum == 0.0f ? acc : acc / lsum;
        store_elem(out, b * os[0] + h * os[1] + s * os[2] + j, res, out_dt);
      }
    }
    free(qv);
    free(kf);
    free(vf);
    free(o);
    free(part);
    free(tmp);
  }
}

int oracle_version(void) { return 1; }
