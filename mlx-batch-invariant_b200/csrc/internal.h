// Host-side interfaces between the translation units of libbi.so.
#pragma once

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

// Fixed tile constants of the tensor-core route (bf16 / fp16).
constexpr int kTcBM = 128;
constexpr int kTcBN = 256;
constexpr int kTcBK = 64;
// Fixed tile constants of the CUDA-core route.
constexpr int kSimtBM = 128;
constexpr int kSimtBN = 128;
constexpr int kSimtBK = 8;

int launch_gemm_tc(const GemmArgs& g, cudaStream_t stream);
int launch_gemm_simt(const GemmArgs& g, cudaStream_t stream);
int launch_sdpa(const SdpaArgs& s, cudaStream_t stream);

// Device error words, one per translation unit; read and optionally clear.
unsigned read_error_gemm_tc(bool clear);
unsigned read_error_sdpa(bool clear);

// Per-thread message for bi_last_error().
int set_error(int status, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);

// Current device's SM count and compute capability (cached per device).
int device_sm_count();
int device_cc_major();

}  // namespace bi
