// Split-K GEMM for callers that cannot allocate device memory.
//
// Some hosts give this library device buffers but forbid it from allocating
// its own: a caller that manages all GPU memory through its own pool (so a
// cudaMalloc would bypass its accounting or fail against its reservation), or
// code that runs where an allocation would synchronise the device. For them,
// omg_gemm_splitk_noalloc runs the split-K tensor-core GEMM with its partial
// slabs and its status word in one file-scope __device__ array instead of in
// memory it allocates.
//
// Limits and sharing:
//  * The array holds kNoAllocScratchBytes (32 MiB) on every GPU that loads
//    the library, for as long as the library stays loaded. The first 256
//    bytes are the status word; the rest holds splits x m x n f32 partials,
//    so splits * m * round_up(n, 4) * 4 must fit in 32 MiB - 256 bytes.
//  * Every call uses the same array and leaves its contents behind; the
//    status word is cleared at the start of each call, and each slab element
//    is written before it is read. Calls whose work overlaps on the GPU (two
//    host threads, or two streams, on one device) race on the array.
//  * The first call on a device looks up the array's device address there
//    (cudaGetSymbolAddress) and sets the kernels' shared-memory limits.
//  * Every call reads the status word back and synchronises `stream` before
//    it returns, so it must never be called while that stream (or, in the
//    global capture mode, any stream) is being captured into a CUDA graph.
//  * The caller's current device is restored before the call returns.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "capi_util.h"
#include "gemm.cuh"
#include "omg_b200.h"

namespace omg {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr size_t kNoAllocHeader = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
uint8_t* g_scratch_ptr[kMaxDevices] = {};

// The array's address on `device` (the current device); looked up once.
uint8_t* scratch_on(int device) {
  std::lock_guard<std::mutex> g(g_setup_mu);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    gemm_setup_device();
    g_scratch_ptr[device] = static_cast<uint8_t*>(p);
  }
  return g_scratch_ptr[device];
}

// out[r, c] = sum over slabs z of part[z, r, c], slabs added in order.
__global__ void sum_slabs(const float* __restrict__ part, int splits, size_t slab, int m, int n,
                          int ldp, float* __restrict__ out, int ldo) {
  const size_t total = static_cast<size_t>(m) * n;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / n, c = i % n;
    float s = part[r * ldp + c];
    for (int z = 1; z < splits; ++z) s += part[z * slab + r * ldp + c];
    out[r * ldo + c] = s;
  }
}

// Makes `device` current for the scope of a call and puts the caller's
// current device back on every exit path.
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int device) {
    CUDA_TRY(cudaGetDevice(&prev));
    if (prev != device) CUDA_TRY(cudaSetDevice(device));
  }
  ~DeviceScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace omg

using namespace omg;

extern "C" int omg_gemm_splitk_noalloc(int device, const void* x_f16, int m, int k, int lda,
                                       const void* w_f16, int n, int splits, float* out, int ldo,
                                       void* stream) {
  return guarded([&]() -> int {
    if (!x_f16 || !w_f16 || !out) fail("omg_gemm_splitk_noalloc: null device pointer");
    if (m <= 0 || n <= 0 || k <= 0) fail("omg_gemm_splitk_noalloc: empty problem");
    if (device < 0 || device >= kMaxDevices) fail("omg_gemm_splitk_noalloc: device %d", device);
    if (ldo < n) fail("omg_gemm_splitk_noalloc: ldo %d < n %d", ldo, n);
    if (lda < k) fail("omg_gemm_splitk_noalloc: lda %d < k %d", lda, k);
    const int kb = (k + 63) / 64;
    if (splits < 1 || splits > kb)
      fail("omg_gemm_splitk_noalloc: splits %d outside 1..%d for K %d", splits, kb, k);
    const int ldp = (n + 3) / 4 * 4;
    const size_t need = static_cast<size_t>(splits) * m * ldp * 4;
    if (need > kNoAllocScratchBytes - kNoAllocHeader)
      fail("omg_gemm_splitk_noalloc: %d x %d x %d f32 partials need %zu bytes; the static "
           "scratch holds %zu",
           splits, m, n, need, kNoAllocScratchBytes - kNoAllocHeader);
    DeviceScope on(device);
    uint8_t* scratch = scratch_on(device);
    auto* status = reinterpret_cast<uint32_t*>(scratch);
    auto* part = reinterpret_cast<float*>(scratch + kNoAllocHeader);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GemmPlan plan;
    char err[256];
    if (!gemm_plan(&plan, x_f16, m, lda, w_f16, n, n, k, kEpiF32, 128, splits, err, sizeof err))
      fail("omg_gemm_splitk_noalloc: %s", err);
    if (plan.s.splits != splits)
      fail("omg_gemm_splitk_noalloc: %d splits leave an empty K slab for K %d", splits, k);
    CUDA_TRY(cudaMemsetAsync(status, 0, 4, s));
    const size_t slab = static_cast<size_t>(m) * ldp;
    gemm_run(plan, m, part, ldp, slab, status, s);
    sum_slabs<<<148 * 4, 256, 0, s>>>(part, splits, slab, m, n, ldp, out, ldo);
    CUDA_TRY(cudaGetLastError());
    uint32_t st = 0;
    CUDA_TRY(cudaMemcpyAsync(&st, status, 4, cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    if (st) fail("omg_gemm_splitk_noalloc: a kernel gave up waiting (device status %u)", st);
    return 0;
  });
}
