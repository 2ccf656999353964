// exb_linear_g128_noalloc: the group-128 exact linear (same result as exb_linear_g128) for
// callers that cannot allocate device memory.
//
// Who needs it: hosts that fix their device-memory budget when they start (a serving process that
// reserves all of HBM for weights and KV caches, or a plugin host that owns the allocator and
// forbids its plugins from calling cudaMalloc), and code that runs where an allocation is not
// allowed or would stall other work (cudaMalloc/cudaFree synchronise the device).  Such callers
// can pass inputs and outputs but cannot provide the scratch buffer exb_linear_g128 needs for the
// quantised activation rows.
//
// Here the scratch is a file-scope __device__ array of fixed size, so every GPU that loads this
// library holds EXB_NOALLOC_SCRATCH_BYTES (24 MiB + 16 KiB) until the process exits: the int16
// rows and their shifts, and the two int8 digit planes the tensor-core GEMM reads.  Limits:
// R * K <= EXB_NOALLOC_MAX_XQ int16 activations, R <= EXB_NOALLOC_MAX_ROWS rows and K <= 25600
// (four int16 rows of K staged in one CTA's shared memory by the GEMV); larger requests are
// rejected with EXB_EINVAL and a message, nothing is launched.  From 16 rows, when N is a multiple
// of 128, the linear runs on the tcgen05 GEMM (one pass over the weights); otherwise on the
// CUDA-core GEMV, one pass over the weights per 4 rows.
//
// The array is shared by every call on a device and keeps the last call's contents.  Each call
// overwrites the parts it reads before reading them (the int16 rows, their shifts, the digit
// planes with their zero padding), so nothing has to start at zero; but two calls whose GPU work
// overlaps (different streams, no ordering) race on the array and give wrong results -- order
// such calls on one stream or with events.
//
// Host code may not pass the array's name to a kernel: on the host it is only a stand-in symbol.
// The device address is looked up once per device with cudaGetSymbolAddress, with that device
// current, on the first call made on that device; make that first call before any stream capture
// on the device.  No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>
#include <string>

#include "common.cuh"
#include "exactb200.h"
#include "exb_internal.h"

// EXB_NOALLOC_MAX_XQ (R * K int16 activations) and EXB_NOALLOC_MAX_ROWS (R) come from exactb200.h
#define EXB_NOALLOC_XQ_BYTES ((size_t)EXB_NOALLOC_MAX_XQ * 2)
#define EXB_NOALLOC_XS_BYTES ((size_t)EXB_NOALLOC_MAX_ROWS * 4)
#define EXB_NOALLOC_DIGIT_BYTES ((size_t)EXB_NOALLOC_MAX_XQ * 4)   // 2 planes x (R padded to 128) x K
#define EXB_NOALLOC_SCRATCH_BYTES (EXB_NOALLOC_XQ_BYTES + EXB_NOALLOC_XS_BYTES + EXB_NOALLOC_DIGIT_BYTES)
#define EXB_NOALLOC_MAX_K 25600

static __device__ __align__(256) unsigned char g_noalloc_scratch[EXB_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};
int fail(int code, const std::string& msg) {
  exb::set_last_error(msg);             // reported by exb_last_error()
  return code;
}
}  // namespace

// device address of the scratch array on the current device (looked up once per device)
static cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

extern "C" int exb_linear_g128_noalloc(const int64_t* x, int R, int K, const int8_t* w_NK, const int32_t* M_NG,
                                       const int64_t* bias, int N, int64_t* y, int64_t* tot_out, void* stream) {
  using namespace exb;
  if (!x || !w_NK || !M_NG || !y || R <= 0 || K <= 0 || N <= 0 || K % 128)
    return fail(EXB_EINVAL, "exb_linear_g128_noalloc: bad arguments (K % 128 == 0 required)");
  if ((long long)R * K > EXB_NOALLOC_MAX_XQ || R > EXB_NOALLOC_MAX_ROWS)
    return fail(EXB_EINVAL, "exb_linear_g128_noalloc: R * K = " + std::to_string((long long)R * K) + " with R = " +
                                std::to_string(R) + " exceeds the fixed scratch (R * K <= " +
                                std::to_string(EXB_NOALLOC_MAX_XQ) + ", R <= " + std::to_string(EXB_NOALLOC_MAX_ROWS) +
                                "); use exb_linear_g128 with caller-provided scratch");
  if (K > EXB_NOALLOC_MAX_K)
    return fail(EXB_EINVAL, "exb_linear_g128_noalloc: K = " + std::to_string(K) + " exceeds " +
                                std::to_string(EXB_NOALLOC_MAX_K) + " (four int16 rows of K per GEMV CTA)");
  if ((uintptr_t)w_NK & 15) return fail(EXB_EINVAL, "exb_linear_g128_noalloc: w must be 16-byte aligned");
  if ((uintptr_t)x & 15) return fail(EXB_EINVAL, "exb_linear_g128_noalloc: x must be 16-byte aligned");
  if ((uintptr_t)M_NG & 3) return fail(EXB_EINVAL, "exb_linear_g128_noalloc: M must be 4-byte aligned");
  if (((uintptr_t)y | (uintptr_t)tot_out | (uintptr_t)bias) & 7)
    return fail(EXB_EINVAL, "exb_linear_g128_noalloc: y, tot and bias must be 8-byte aligned");
  void* base = nullptr;
  cudaError_t e = noalloc_scratch(&base);
  if (e != cudaSuccess)
    return fail(EXB_ECUDA, std::string("exb_linear_g128_noalloc: cudaGetSymbolAddress -> ") + cudaGetErrorString(e));
  int16_t* xq = static_cast<int16_t*>(base);
  int32_t* xs = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(base) + EXB_NOALLOC_XQ_BYTES);
  void* digits = static_cast<unsigned char*>(base) + EXB_NOALLOC_XQ_BYTES + EXB_NOALLOC_XS_BYTES;
  cudaStream_t st = (cudaStream_t)stream;
  // the kernels read the (N, K/128) scales 4 bytes at a time: any row pitch >= K/128 works
  LinW L;
  L.w = w_NK; L.Mg = M_NG; L.ldm = K / 128; L.b = bias; L.N = N; L.K = K;
  // xq, s = qrow(x) for every row (exact_llm.py:41-46); overwrites the rows it later reads
  e = launch_quant(x, K, R, K, xq, K, xs, st, false);
  if (e == cudaSuccess && R >= TC_MIN_ROWS && gemm_tc_digit_bytes(R, K) <= EXB_NOALLOC_DIGIT_BYTES &&
      gemm_tc_supported(L, EPI_STORE)) {
    // tcgen05 path: both int8 digit planes (rows padded with zeros) in the fixed array
    e = launch_digits(xq, K, R, K, digits, st);
    if (e == cudaSuccess) e = launch_gemm_tc(digits, R, L, xs, EPI_STORE, y, N, tot_out, nullptr, N, nullptr, nullptr, st);
  } else {
    for (int r0 = 0; e == cudaSuccess && r0 < R; r0 += 4) {
      GemvArgs g;
      g.xq = xq + (size_t)r0 * K; g.xs = xs + r0; g.ldx = K;
      g.L = L;
      g.R = R - r0 < 4 ? R - r0 : 4;
      g.epi = EPI_STORE; g.out = y + (size_t)r0 * N; g.ldo = N;
      g.raw = tot_out ? tot_out + (size_t)r0 * N : nullptr; g.ldr = N;
      e = launch_gemv(g, st, false);
    }
  }
  if (e != cudaSuccess) return fail(EXB_ECUDA, std::string("exb_linear_g128_noalloc: launch -> ") + cudaGetErrorString(e));
  return EXB_OK;
}
