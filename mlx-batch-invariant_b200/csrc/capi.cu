// extern "C" entry points of libbi.so (declared in include/bi.h): argument
// validation, route selection and error reporting.  The kernels live in
// gemm_tcgen05.cu, gemm_simt.cu and sdpa.cu.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "internal.h"

namespace bi {

static thread_local char g_msg[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return BI_OK;
  return set_error(BI_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

namespace {
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int> g_cc_major[kMaxDevices];

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int elem_size(int dtype) { return dtype == BI_F32 ? 4 : 2; }
}  // namespace

int device_sm_count() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int v = g_sm_count[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
      v = 148;
    }
    g_sm_count[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

int device_cc_major() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return -1;
  int v = g_cc_major[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
      return -1;
    }
    g_cc_major[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// The GEMM route for (dtype, K, N, layout).  Never a function of M.
static int gemm_route(int dtype, int64_t K, int64_t N, int b_is_nk) {
  if (dtype == BI_F32) return BI_ROUTE_SIMT;
  if (K <= 0 || K % 8 != 0) return BI_ROUTE_SIMT;
  if (!b_is_nk && N % 8 != 0) return BI_ROUTE_SIMT;
  return BI_ROUTE_TCGEN05;
}

// Peer access from device `cur` (current) to `peer`'s memory, enabled if the hardware
// allows it; "already enabled" counts as success.  A pair found usable is remembered.
static int ensure_peer_access(int cur, int peer) {
  static std::mutex mu;
  static bool ok[kMaxDevices][kMaxDevices] = {};
  if (cur < 0 || cur >= kMaxDevices || peer < 0 || peer >= kMaxDevices) {
    return set_error(BI_ERR_INVALID, "device ordinal %d out of range", cur < 0 ? cur : peer);
  }
  std::lock_guard<std::mutex> lock(mu);
  if (ok[cur][peer]) return BI_OK;
  int can = 0;
  cudaError_t e = cudaDeviceCanAccessPeer(&can, cur, peer);
  if (e != cudaSuccess) return cuda_status(e, "cudaDeviceCanAccessPeer");
  if (!can) {
    return set_error(BI_ERR_UNSUPPORTED, "device %d cannot access device %d's memory (no peer "
                     "access between them)", cur, peer);
  }
  e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();  // the answer is success; do not leave it as the last error
  } else if (e != cudaSuccess) {
    return cuda_status(e, "cudaDeviceEnablePeerAccess");
  }
  ok[cur][peer] = true;
  return BI_OK;
}

// Shapes the fp32 tensor-core route takes: TMA needs 16-byte row strides.
static bool tf32x3_shape_ok(int64_t K, int64_t N, int b_is_nk) {
  return K > 0 && K % 4 == 0 && (b_is_nk || N % 4 == 0);
}

static int check_device() {
  const int cc = device_cc_major();
  if (cc < 0) return set_error(BI_ERR_NO_DEVICE, "no CUDA device is current");
  if (cc != 10) {
    return set_error(BI_ERR_NO_DEVICE, "libbi.so is built for sm_100a; current device is sm_%d*",
                     cc);
  }
  return BI_OK;
}

}  // namespace bi

using namespace bi;

extern "C" {

int bi_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, const void* bias, void* out,
            int64_t ldo, int64_t M, int64_t N, int64_t K, int b_is_nk, float alpha, float beta,
            int dtype, void* stream) {
  g_msg[0] = '\0';
  if (dtype != BI_F32 && dtype != BI_F16 && dtype != BI_BF16) {
    return set_error(BI_ERR_INVALID, "unknown dtype %d", dtype);
  }
  if (M < 0 || N < 0 || K < 0) return set_error(BI_ERR_INVALID, "negative dimension");
  if (M == 0 || N == 0) return BI_OK;
  if (out == nullptr) return set_error(BI_ERR_INVALID, "out is null");
  if (K > 0 && (a == nullptr || b == nullptr)) return set_error(BI_ERR_INVALID, "a or b is null");
  if (lda < K || ldo < N || ldb < (b_is_nk ? K : N)) {
    return set_error(BI_ERR_INVALID, "leading dimension smaller than the row");
  }
  int st = check_device();
  if (st) return st;

  GemmArgs g{a, lda, b, ldb, bias, out, ldo, M, N, K, b_is_nk ? 1 : 0, alpha, beta, dtype};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gemm_route(dtype, K, N, b_is_nk) == BI_ROUTE_TCGEN05) {
    if (!aligned16(a) || !aligned16(b) || lda % 8 != 0 || ldb % 8 != 0) {
      return set_error(BI_ERR_MISALIGNED,
                       "tensor-core route needs 16-byte aligned a/b and row strides that are "
                       "multiples of 8 elements");
    }
    return launch_gemm_tc(g, s);
  }
  return launch_gemm_simt(g, s);
}

int bi_gemm_tf32x3(const void* a, int64_t lda, const void* b, int64_t ldb, const void* bias,
                   void* out, int64_t ldo, int64_t M, int64_t N, int64_t K, int b_is_nk,
                   float alpha, float beta, void* stream) {
  g_msg[0] = '\0';
  if (M < 0 || N < 0 || K < 0) return set_error(BI_ERR_INVALID, "negative dimension");
  if (M == 0 || N == 0) return BI_OK;
  if (out == nullptr) return set_error(BI_ERR_INVALID, "out is null");
  if (K > 0 && (a == nullptr || b == nullptr)) return set_error(BI_ERR_INVALID, "a or b is null");
  if (lda < K || ldo < N || ldb < (b_is_nk ? K : N)) {
    return set_error(BI_ERR_INVALID, "leading dimension smaller than the row");
  }
  if (!tf32x3_shape_ok(K, N, b_is_nk)) {
    return set_error(BI_ERR_UNSUPPORTED,
                     "the tf32x3 route needs K %% 4 == 0 (and N %% 4 == 0 for a (K, N) b)");
  }
  if (!aligned16(a) || !aligned16(b) || lda % 4 != 0 || ldb % 4 != 0) {
    return set_error(BI_ERR_MISALIGNED,
                     "the tf32x3 route needs 16-byte aligned a/b and row strides that are "
                     "multiples of 4 elements");
  }
  int st = check_device();
  if (st) return st;
  GemmArgs g{a, lda, b, ldb, bias, out, ldo, M, N, K, b_is_nk ? 1 : 0, alpha, beta, BI_F32};
  return launch_gemm_tf32x3(g, static_cast<cudaStream_t>(stream));
}

int bi_gemm_route(int dtype, int64_t K, int64_t N, int b_is_nk, int* route, int* bm, int* bn,
                  int* bk) {
  if (dtype != BI_F32 && dtype != BI_F16 && dtype != BI_BF16) {
    return set_error(BI_ERR_INVALID, "unknown dtype %d", dtype);
  }
  const int r = gemm_route(dtype, K, N, b_is_nk);
  if (route) *route = r;
  if (bm) *bm = r == BI_ROUTE_TCGEN05 ? kTcBM : kSimtBM;
  if (bn) *bn = r == BI_ROUTE_TCGEN05 ? kTcBN : kSimtBN;
  if (bk) *bk = r == BI_ROUTE_TCGEN05 ? kTcBK : kSimtBK;
  return BI_OK;
}

int bi_sdpa(const void* q, const int64_t q_strides[3], const void* k, const int64_t k_strides[2],
            const void* v, const int64_t v_strides[2], const void* mask,
            const int64_t mask_strides[3], int mask_mode, int64_t causal_offset,
            const void* sinks, float scale, int64_t B, int64_t H, int64_t Hkv, int64_t qL,
            int64_t N, int64_t D, int64_t V, int dtype, void* out, const int64_t out_strides[3],
            void* stream) {
  g_msg[0] = '\0';
  if (dtype != BI_F32 && dtype != BI_F16 && dtype != BI_BF16) {
    return set_error(BI_ERR_INVALID, "unknown dtype %d", dtype);
  }
  if (B < 0 || H < 0 || Hkv < 0 || qL < 0 || N < 0 || D <= 0 || V <= 0) {
    return set_error(BI_ERR_INVALID, "negative or empty dimension");
  }
  if (Hkv == 0 || H % Hkv != 0) return set_error(BI_ERR_INVALID, "H must be a multiple of Hkv");
  if (D % 32 != 0 || V % 32 != 0) {
    return set_error(BI_ERR_INVALID, "head dimensions must be multiples of 32");
  }
  const bool f32 = dtype == BI_F32;
  if ((f32 && (D > 384 || V > 384 || D + V > 768)) || (!f32 && (D > 640 || V > 640))) {
    return set_error(BI_ERR_UNSUPPORTED,
                     "head dims D=%lld V=%lld are not built (D, V <= 640 for 16-bit types; "
                     "D, V <= 384 and D + V <= 768 for float32)",
                     static_cast<long long>(D), static_cast<long long>(V));
  }
  if (mask_mode < 0 || mask_mode > 2) return set_error(BI_ERR_INVALID, "mask_mode must be 0..2");
  if (B == 0 || H == 0 || qL == 0) return BI_OK;
  if (!q_strides || !k_strides || !v_strides || !out_strides) {
    return set_error(BI_ERR_INVALID, "stride array is null");
  }
  if (mask_mode == 2 && (mask == nullptr || mask_strides == nullptr)) {
    return set_error(BI_ERR_INVALID, "mask_mode 2 needs a mask and its strides");
  }
  if (B > INT32_MAX || H > INT32_MAX || qL > INT32_MAX || N > INT32_MAX) {
    return set_error(BI_ERR_UNSUPPORTED, "dimensions above 2^31 are not supported");
  }
  if (q == nullptr || out == nullptr || (N > 0 && (k == nullptr || v == nullptr))) {
    return set_error(BI_ERR_INVALID, "q, k, v or out is null");
  }
  const int64_t vec = 16 / elem_size(dtype);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || q_strides[0] % vec ||
      q_strides[1] % vec || q_strides[2] % vec || k_strides[0] % vec || k_strides[1] % vec ||
      v_strides[0] % vec || v_strides[1] % vec) {
    return set_error(BI_ERR_MISALIGNED,
                     "q, k, v must be 16-byte aligned with strides that are multiples of 16 bytes");
  }
  int st = check_device();
  if (st) return st;

  SdpaArgs a;
  a.q = q;
  for (int i = 0; i < 3; ++i) a.qs[i] = q_strides[i];
  a.k = k;
  a.ks[0] = k_strides[0];
  a.ks[1] = k_strides[1];
  a.v = v;
  a.vs[0] = v_strides[0];
  a.vs[1] = v_strides[1];
  a.mask = mask_mode == 2 ? mask : nullptr;
  for (int i = 0; i < 3; ++i) a.ms[i] = mask_mode == 2 ? mask_strides[i] : 0;
  a.mask_mode = mask_mode;
  a.causal_offset = causal_offset;
  a.sinks = sinks;
  a.scale = scale;
  a.B = B;
  a.H = H;
  a.Hkv = Hkv;
  a.qL = qL;
  a.N = N;
  a.D = D;
  a.V = V;
  a.dtype = dtype;
  a.out = out;
  for (int i = 0; i < 3; ++i) a.os[i] = out_strides[i];
  return launch_sdpa(a, static_cast<cudaStream_t>(stream));
}

int bi_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
  g_msg[0] = '\0';
  if (bytes <= 0 || ptr == nullptr || ipc_handle == nullptr) {
    return set_error(BI_ERR_INVALID, "bi_peer_alloc: bad arguments");
  }
  int st = check_device();
  if (st) return st;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return cuda_status(e, "cudaMalloc(peer buffer)");
  e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e, "peer buffer set-up");
  }
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return BI_OK;
}

int bi_peer_open(const void* ipc_handle, void** ptr) {
  g_msg[0] = '\0';
  if (ipc_handle == nullptr || ptr == nullptr) return set_error(BI_ERR_INVALID, "bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess),
                     "cudaIpcOpenMemHandle");
}

int bi_peer_close(void* ptr) {
  g_msg[0] = '\0';
  return cuda_status(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

int bi_peer_free(void* ptr) {
  g_msg[0] = '\0';
  return cuda_status(cudaFree(ptr), "cudaFree(peer buffer)");
}

// Validates the rank set and (when given) the staging areas and the column partition.
static int gather_args(void* const* stages, void* const* flags, const int64_t* cols, int rank,
                       int world, uint32_t epoch, GatherArgs* x) {
  if (world < 1 || world > BI_MAX_PEERS || rank < 0 || rank >= world || flags == nullptr) {
    return set_error(BI_ERR_INVALID, "rank %d / world %d outside [0, %d)", rank, world,
                     BI_MAX_PEERS);
  }
  *x = GatherArgs{};
  for (int r = 0; r < world; ++r) {
    if (flags[r] == nullptr || (stages != nullptr && stages[r] == nullptr)) {
      return set_error(BI_ERR_INVALID, "null peer pointer for rank %d", r);
    }
    x->flags[r] = static_cast<uint32_t*>(flags[r]);
    x->stages[r] = stages != nullptr ? stages[r] : nullptr;
  }
  x->local = x->flags[rank];
  if (cols != nullptr) {
    if (cols[0] != 0) return set_error(BI_ERR_INVALID, "cols[0] must be 0");
    for (int r = 0; r <= world; ++r) {
      if (r > 0 && cols[r] < cols[r - 1]) {
        return set_error(BI_ERR_INVALID, "cols must be nondecreasing");
      }
      if (cols[r] % 8 != 0) {
        return set_error(BI_ERR_MISALIGNED, "column bounds must be multiples of 8");
      }
      x->cols[r] = cols[r];
    }
  }
  x->rank = rank;
  x->world = world;
  x->epoch = epoch;
  return BI_OK;
}

int bi_peer_barrier(void* const* flags, int rank, int world, uint32_t epoch, void* stream) {
  g_msg[0] = '\0';
  GatherArgs x;
  int st = gather_args(nullptr, flags, nullptr, rank, world, epoch, &x);
  if (st) return st;
  st = check_device();
  if (st) return st;
  return launch_peer_barrier(x, static_cast<cudaStream_t>(stream));
}

static int gemm_allgather(const void* a, int64_t lda, const void* b, int64_t ldb,
                          const void* bias, void* out, int64_t ldo, void* const* stages,
                          const int64_t* cols, int64_t M, int64_t K, int b_is_nk, float alpha,
                          float beta, int dtype, void* const* flags, int rank, int world,
                          uint32_t epoch, void* stream, bool unpack,
                          uint32_t* local = nullptr) {
  g_msg[0] = '\0';
  if (dtype != BI_F16 && dtype != BI_BF16) {
    return set_error(BI_ERR_UNSUPPORTED, "the fused all-gather takes fp16 or bf16");
  }
  if (M < 0 || K < 0) return set_error(BI_ERR_INVALID, "negative size");
  if (stages == nullptr || cols == nullptr) {
    return set_error(BI_ERR_INVALID, "stages and cols must not be null");
  }
  GatherArgs x;
  int st = gather_args(stages, flags, cols, rank, world, epoch, &x);
  if (st) return st;
  if (local != nullptr) x.local = local;
  const int64_t n_total = x.cols[world];
  const int64_t n_local = x.cols[rank + 1] - x.cols[rank];
  if (ldo % 8 != 0 || ldo < n_total) {
    return set_error(BI_ERR_MISALIGNED, "ldo must be a multiple of 8 and at least cols[world]");
  }
  st = check_device();
  if (st) return st;
  if (M > 0 && n_total > 0) {
    if (!aligned16(out)) return set_error(BI_ERR_MISALIGNED, "out must be 16-byte aligned");
    for (int r = 0; r < world; ++r) {
      if (!aligned16(stages[r])) return set_error(BI_ERR_MISALIGNED, "staging areas must be aligned");
    }
  }
  if (n_local > 0 && M > 0) {
    if (gemm_route(dtype, K, n_local, b_is_nk) != BI_ROUTE_TCGEN05) {
      return set_error(BI_ERR_UNSUPPORTED, "the fused all-gather needs the tensor-core route");
    }
    if (!aligned16(a) || !aligned16(b) || lda % 8 != 0 || ldb % 8 != 0 || lda < K ||
        ldb < (b_is_nk ? K : n_local)) {
      return set_error(BI_ERR_MISALIGNED, "a/b must be 16-byte aligned with 8-element strides");
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Entry barrier: every rank has finished the work queued before this call (the
  // unpack that read the previous contents of its staging area) before any rank
  // writes into it.
  st = launch_peer_barrier(x, s);
  if (st) return st;
  void* out_shard = out != nullptr ? static_cast<uint16_t*>(out) + x.cols[rank] : nullptr;
  GemmArgs g{a, lda, b, ldb, bias, out_shard, ldo, M, n_local, K, b_is_nk ? 1 : 0,
             alpha, beta, dtype};
  return launch_gemm_tc_allgather(g, x, out, s, unpack);
}

int bi_gemm_allgather(const void* a, int64_t lda, const void* b, int64_t ldb, const void* bias,
                      void* out, int64_t ldo, void* const* stages, const int64_t* cols,
                      int64_t M, int64_t K, int b_is_nk, float alpha, float beta, int dtype,
                      void* const* flags, int rank, int world, uint32_t epoch, void* stream) {
  return gemm_allgather(a, lda, b, ldb, bias, out, ldo, stages, cols, M, K, b_is_nk, alpha, beta,
                        dtype, flags, rank, world, epoch, stream, true);
}

int bi_gemm_allgather_deferred(const void* a, int64_t lda, const void* b, int64_t ldb,
                               const void* bias, void* out, int64_t ldo, void* const* stages,
                               const int64_t* cols, int64_t M, int64_t K, int b_is_nk,
                               float alpha, float beta, int dtype, void* const* flags, int rank,
                               int world, uint32_t epoch, void* stream) {
  return gemm_allgather(a, lda, b, ldb, bias, out, ldo, stages, cols, M, K, b_is_nk, alpha, beta,
                        dtype, flags, rank, world, epoch, stream, false);
}

int bi_gather_unpack(void* out, int64_t ldo, void* const* stages, const int64_t* cols, int64_t M,
                     int rank, int world, int dtype, void* stream) {
  g_msg[0] = '\0';
  if (dtype != BI_F16 && dtype != BI_BF16) {
    return set_error(BI_ERR_UNSUPPORTED, "the fused all-gather takes fp16 or bf16");
  }
  if (M < 0) return set_error(BI_ERR_INVALID, "negative size");
  if (stages == nullptr || cols == nullptr) {
    return set_error(BI_ERR_INVALID, "stages and cols must not be null");
  }
  if (world < 1 || world > BI_MAX_PEERS || rank < 0 || rank >= world) {
    return set_error(BI_ERR_INVALID, "rank %d / world %d outside [0, %d)", rank, world,
                     BI_MAX_PEERS);
  }
  GatherArgs x{};
  if (cols[0] != 0) return set_error(BI_ERR_INVALID, "cols[0] must be 0");
  for (int r = 0; r <= world; ++r) {
    if (r > 0 && cols[r] < cols[r - 1]) return set_error(BI_ERR_INVALID, "cols must be nondecreasing");
    if (cols[r] % 8 != 0) return set_error(BI_ERR_MISALIGNED, "column bounds must be multiples of 8");
    x.cols[r] = cols[r];
  }
  if (stages[rank] == nullptr) return set_error(BI_ERR_INVALID, "this rank's staging area is null");
  x.stages[rank] = stages[rank];
  x.rank = rank;
  x.world = world;
  if (ldo % 8 != 0 || ldo < x.cols[world]) {
    return set_error(BI_ERR_MISALIGNED, "ldo must be a multiple of 8 and at least cols[world]");
  }
  if (M > 0 && x.cols[world] > 0 && (out == nullptr || !aligned16(out) || !aligned16(stages[rank]))) {
    return set_error(BI_ERR_MISALIGNED, "out and the staging area must be 16-byte aligned");
  }
  int st = check_device();
  if (st) return st;
  return launch_gather_unpack(x, out, ldo, M, static_cast<cudaStream_t>(stream));
}

int bi_gemm_allgather_static(const void* a, int64_t lda, const void* b, int64_t ldb,
                             const void* bias, void* out, int64_t ldo, void* const* stages,
                             const int64_t* cols, int64_t M, int64_t K, int b_is_nk, float alpha,
                             float beta, int dtype, const int* devices, int rank, int world,
                             uint32_t epoch, void* stream) {
  g_msg[0] = '\0';
  if (world < 1 || world > BI_MAX_PEERS) {
    return set_error(BI_ERR_INVALID,
                     "bi_gemm_allgather_static: world %d outside [1, %d] -- the exchange "
                     "flags hold at most %d ranks",
                     world, BI_MAX_PEERS, BI_MAX_PEERS);
  }
  if (devices == nullptr) return set_error(BI_ERR_INVALID, "devices is null");
  if (rank < 0 || rank >= world) return set_error(BI_ERR_INVALID, "rank outside [0, world)");
  if (stages == nullptr) return set_error(BI_ERR_INVALID, "stages is null");
  // One rank per device: two ranks on one device would share its counters (the CTA
  // counter and the call count), and one rank's counter reset could land in the
  // other's call.
  for (int r = 0; r < world; ++r) {
    for (int r2 = r + 1; r2 < world; ++r2) {
      if (devices[r] == devices[r2]) {
        return set_error(BI_ERR_INVALID,
                         "bi_gemm_allgather_static: ranks %d and %d are both on device %d; "
                         "the static counters hold one rank per device",
                         r, r2, devices[r]);
      }
    }
  }
  for (int r = 0; r < world; ++r) {
    if (stages[r] == nullptr || !aligned16(stages[r])) {
      return set_error(BI_ERR_MISALIGNED, "exchange area of rank %d is null or not 16-byte "
                       "aligned", r);
    }
  }
  int st = check_device();
  if (st) return st;
  // The local GEMM counts its CTAs in the array of the device it runs on.
  const int cur = current_device();
  if (devices[rank] != cur) {
    return set_error(BI_ERR_INVALID,
                     "bi_gemm_allgather_static: devices[%d] = %d but device %d is current; "
                     "call each rank with its own device current",
                     rank, devices[rank], cur);
  }
  // The kernels store into every other rank's exchange area: this device must reach
  // each of those devices' memory.
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    st = ensure_peer_access(cur, devices[r]);
    if (st) return st;
  }
  void* local = nullptr;
  st = static_flag_block(cur, &local);
  if (st) return st;
  // Each exchange area starts with the rank's flag block; its staging area follows.
  void* flags[BI_MAX_PEERS] = {};
  void* data[BI_MAX_PEERS] = {};
  for (int r = 0; r < world; ++r) {
    flags[r] = stages[r];
    data[r] = static_cast<uint8_t*>(stages[r]) + BI_PEER_FLAG_BYTES;
  }
  // The array keeps the previous call's contents; the CTA counter must start at zero.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(static_cast<uint32_t*>(local) + kFlagCounter, 0,
                                  sizeof(uint32_t), s);
  if (e != cudaSuccess) return cuda_status(e, "clearing the static CTA counter");
  return gemm_allgather(a, lda, b, ldb, bias, out, ldo, data, cols, M, K, b_is_nk, alpha, beta,
                        dtype, flags, rank, world, epoch, stream, true,
                        static_cast<uint32_t*>(local));
}

int bi_rope_kv(const void* qkv, int64_t B, int64_t L, int64_t hq, int64_t hk, int64_t hd,
               const float* cos_tab, const float* sin_tab, int64_t p0, const int64_t* pos,
               int64_t n_pos, void* q_out, void* k_cache, void* v_cache,
               const int64_t cache_strides[3], int dtype, void* stream) {
  g_msg[0] = '\0';
  if (dtype != BI_F32 && dtype != BI_F16 && dtype != BI_BF16) {
    return set_error(BI_ERR_INVALID, "unknown dtype %d", dtype);
  }
  if (B < 0 || L < 0 || hq < 0 || hk < 0 || hd <= 0 || hd % 2 != 0 || p0 < 0) {
    return set_error(BI_ERR_INVALID, "bad rope sizes (hd must be even and positive)");
  }
  if (B * L * (hq + hk) > 0 &&
      (qkv == nullptr || cos_tab == nullptr || sin_tab == nullptr || cache_strides == nullptr ||
       (hq > 0 && q_out == nullptr) || (hk > 0 && (k_cache == nullptr || v_cache == nullptr)))) {
    return set_error(BI_ERR_INVALID, "null pointer");
  }
  if (n_pos < 0) return set_error(BI_ERR_INVALID, "n_pos must not be negative");
  if (pos == nullptr && p0 + L > n_pos) {
    return set_error(BI_ERR_INVALID, "positions %lld..%lld are past the %lld the tables hold",
                     static_cast<long long>(p0), static_cast<long long>(p0 + L - 1),
                     static_cast<long long>(n_pos));
  }
  int st = check_device();
  if (st) return st;
  RopeArgs a{qkv, B, L, hq, hk, hd, cos_tab, sin_tab, p0, pos, n_pos, q_out, k_cache, v_cache,
             cache_strides != nullptr ? cache_strides[0] : 0,
             cache_strides != nullptr ? cache_strides[1] : 0,
             cache_strides != nullptr ? cache_strides[2] : 0};
  return launch_rope_kv(a, dtype, static_cast<cudaStream_t>(stream));
}

int bi_swiglu(const void* gu, void* out, int64_t M, int64_t I, int dtype, void* stream) {
  g_msg[0] = '\0';
  if (dtype != BI_F32 && dtype != BI_F16 && dtype != BI_BF16) {
    return set_error(BI_ERR_INVALID, "unknown dtype %d", dtype);
  }
  if (M < 0 || I < 0) return set_error(BI_ERR_INVALID, "negative size");
  if (M * I > 0 && (gu == nullptr || out == nullptr)) return set_error(BI_ERR_INVALID, "null pointer");
  int st = check_device();
  if (st) return st;
  return launch_swiglu(gu, out, M, I, dtype, static_cast<cudaStream_t>(stream));
}

const char* bi_status_string(int status) {
  switch (status) {
    case BI_OK: return "ok";
    case BI_ERR_INVALID: return "invalid argument";
    case BI_ERR_UNSUPPORTED: return "unsupported";
    case BI_ERR_MISALIGNED: return "misaligned pointer or stride";
    case BI_ERR_CUDA: return "CUDA error";
    case BI_ERR_TIMEOUT: return "device wait timed out";
    case BI_ERR_NO_DEVICE: return "no suitable CUDA device";
    default: return "unknown status";
  }
}

const char* bi_last_error(void) { return g_msg; }

int bi_device_error(int clear) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "cudaDeviceSynchronize");
  unsigned w = read_error_gemm_tc(clear != 0);
  const unsigned s = read_error_sdpa(clear != 0);
  const unsigned h = read_error_harness(clear != 0);
  const unsigned t = read_error_tf32x3(clear != 0);
  if (w == 0 && s != 0) w = s | (1u << 16);  // sdpa sites are tagged in bit 16
  if (w == 0 && h != 0) w = h | (1u << 17);  // decoder-harness sites in bit 17
  if (w == 0 && t != 0) w = t | (1u << 18);  // fp32 tensor-core GEMM sites in bit 18
  return static_cast<int>(w);
}

int bi_version(void) { return 100; }  // 0.1.0

}  // extern "C"
