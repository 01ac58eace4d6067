// Elementwise steps of the Llama-shaped decoder harness, fused: rotary embedding of q
// and k together with the KV-cache write (one kernel instead of ~18 small ones per
// layer), and SwiGLU (silu(gate) * up).  The reference's harness runs its framework's
// own ops here (bench/bench.py:108-159); these kernels only cut launches.
//
// Every output element comes from its own inputs by the same fp32 operations, each
// rounded, as the torch expressions they replace:
//   rope:   o1 = x1*cos - x2*sin,  o2 = x2*cos + x1*sin   (x = float(t), one rounding
//           per mul / add, then to the storage type), cos/sin from fp32 tables;
//   swiglu: s = to_T(g / (1 + exp(-g)));  out = to_T(float(s) * u).
// Nothing depends on how many rows are in flight, so both are batch-invariant.
#include "common.cuh"
#include "internal.h"

namespace bi {
namespace harness {

// Error site of the rope kernel: a row whose position lies outside [0, n_pos) (the
// position can come from device memory, where the host cannot check it).
constexpr unsigned kSiteRopePosition = 1;
constexpr unsigned kErrReasonRange = 2;

__device__ unsigned g_error_word = 0;

template <typename T>
__global__ void __launch_bounds__(256) rope_kv_kernel(const RopeArgs a) {
  const int64_t half = a.hd / 2;
  const int64_t nheads = a.hq + 2 * a.hk;
  const int64_t total = a.B * a.L * nheads * half;
  const T* qkv = static_cast<const T*>(a.qkv);
  const int64_t base = a.pos != nullptr ? *a.pos : a.p0;
  // Rows past the tables or the caches are not written; the call reports it through
  // the device error word instead.
  if (base < 0 || base + a.L > a.n_pos) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      record_error(&g_error_word, (kSiteRopePosition << 8) | kErrReasonRange);
    }
  }
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx % half;
    int64_t t = idx / half;
    const int64_t h = t % nheads;
    t /= nheads;
    const int64_t l = t % a.L;
    const int64_t b = t / a.L;
    const int64_t pos = base + l;
    if (pos < 0 || pos >= a.n_pos) continue;
    const T* src = qkv + ((b * a.L + l) * nheads + h) * a.hd;
    if (h < a.hq + a.hk) {
      const float c = a.cos_tab[pos * half + i];
      const float sn = a.sin_tab[pos * half + i];
      const float x1 = to_f32(src[i]);
      const float x2 = to_f32(src[i + half]);
      const T o1 = from_f32<T>(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn)));
      const T o2 = from_f32<T>(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn)));
      T* dst = h < a.hq ? static_cast<T*>(a.q_out) + ((b * a.hq + h) * a.L + l) * a.hd
                        : static_cast<T*>(a.k_cache) + b * a.cs0 + (h - a.hq) * a.cs1 +
                              pos * a.cs2;
      dst[i] = o1;
      dst[i + half] = o2;
    } else {
      T* dst = static_cast<T*>(a.v_cache) + b * a.cs0 + (h - a.hq - a.hk) * a.cs1 + pos * a.cs2;
      dst[i] = src[i];
      dst[i + half] = src[i + half];
    }
  }
}

template <typename T>
__device__ __forceinline__ T swiglu1(T g, T u) {
  const float gf = to_f32(g);
  const T s = from_f32<T>(__fdiv_rn(gf, __fadd_rn(1.0f, expf(-gf))));
  return from_f32<T>(__fmul_rn(to_f32(s), to_f32(u)));
}

// gu (M, 2I) = [gate | up] per row, out (M, I).  VEC: I % 8 == 0 and 16-byte aligned
// rows, 8 elements per thread step.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* gu, T* out, int64_t M, int64_t I) {
  static_assert(!VEC || sizeof(T) == 2, "8-element vectors are 16 bytes of 16-bit data");
  const int64_t per = VEC ? 8 : 1;
  const int64_t total = M * I / per;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = idx * per;
    const int64_t m = e / I;
    const int64_t i = e - m * I;
    const T* g = gu + m * 2 * I + i;
    if constexpr (VEC) {
      const uint4 gv = *reinterpret_cast<const uint4*>(g);
      const uint4 uv = *reinterpret_cast<const uint4*>(g + I);
      const T* gp = reinterpret_cast<const T*>(&gv);
      const T* up = reinterpret_cast<const T*>(&uv);
      uint4 ov;
      T* op = reinterpret_cast<T*>(&ov);
#pragma unroll
      for (int j = 0; j < 8; ++j) op[j] = swiglu1<T>(gp[j], up[j]);
      *reinterpret_cast<uint4*>(out + e) = ov;
    } else {
      out[e] = swiglu1<T>(g[0], g[I]);
    }
  }
}

static unsigned grid_for(int64_t work) {
  const int64_t cap = 8LL * device_sm_count();
  const int64_t want = (work + 255) / 256;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace harness

int launch_rope_kv(const RopeArgs& a, int dtype, cudaStream_t stream) {
  const int64_t work = a.B * a.L * (a.hq + 2 * a.hk) * (a.hd / 2);
  if (work == 0) return BI_OK;
  const unsigned g = harness::grid_for(work);
  if (dtype == BI_BF16) {
    harness::rope_kv_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(a);
  } else if (dtype == BI_F16) {
    harness::rope_kv_kernel<__half><<<g, 256, 0, stream>>>(a);
  } else {
    harness::rope_kv_kernel<float><<<g, 256, 0, stream>>>(a);
  }
  return cuda_status(cudaGetLastError(), "rope_kv launch");
}

template <typename T>
static int launch_swiglu_t(const void* gu, void* out, int64_t M, int64_t I, cudaStream_t stream) {
  const T* g = static_cast<const T*>(gu);
  T* o = static_cast<T*>(out);
  if constexpr (sizeof(T) == 2) {
    if (I % 8 == 0 && reinterpret_cast<uintptr_t>(gu) % 16 == 0 &&
        reinterpret_cast<uintptr_t>(out) % 16 == 0) {
      harness::swiglu_kernel<T, true><<<harness::grid_for(M * I / 8), 256, 0, stream>>>(g, o, M, I);
      return cuda_status(cudaGetLastError(), "swiglu launch");
    }
  }
  harness::swiglu_kernel<T, false><<<harness::grid_for(M * I), 256, 0, stream>>>(g, o, M, I);
  return cuda_status(cudaGetLastError(), "swiglu launch");
}

unsigned read_error_harness(bool clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, harness::g_error_word, sizeof(v));
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(harness::g_error_word, &z, sizeof(z));
  }
  return v;
}

int launch_swiglu(const void* gu, void* out, int64_t M, int64_t I, int dtype,
                  cudaStream_t stream) {
  if (M * I == 0) return BI_OK;
  if (dtype == BI_BF16) return launch_swiglu_t<__nv_bfloat16>(gu, out, M, I, stream);
  if (dtype == BI_F16) return launch_swiglu_t<__half>(gu, out, M, I, stream);
  return launch_swiglu_t<float>(gu, out, M, I, stream);
}

}  // namespace bi
