// sp_loss_sums_noalloc: the per-pixel loss sums of sp_read_loss for callers that cannot
// allocate device memory. Some hosts own every byte of the GPU through their own allocator
// (a game engine or another framework with a fixed memory budget), and some run in loops
// where a cudaMalloc / cudaFree, which synchronise the whole device, would stall them; such
// callers pass their input and output buffers and need the library to bring nothing else.
//
// The reduction's scratch (four double partials per block and a completion counter)
// therefore lives in a fixed file-scope device array of 4 * 1024 + 1 doubles (32,776 bytes,
// about 32 KiB), which every GPU that loads this library holds until the process exits.
// That fixes the largest input: SP_NOALLOC_MAX_PIXELS pixels (1024 blocks of 4096).
#include <cstdint>
#include <mutex>

#include "kernels.h"

namespace splat {
namespace {

constexpr int kThreads = 256;
constexpr int kPixelsPerBlock = 4096;
constexpr int kMaxBlocks = (int)(SP_NOALLOC_MAX_PIXELS / kPixelsPerBlock);
constexpr int kMaxDevices = 64;

// Four double partials per block, then the completion counter in the last slot. Shared by
// every call on a device: the partials are overwritten by each call, the counter is
// cleared by each call before its kernel runs, so calls that overlap on the GPU race.
static __device__ __align__(256) double g_scratch[4 * kMaxBlocks + 1];
static_assert(sizeof(g_scratch) == 32776, "the documented scratch size (include/splat.h) is 32,776 bytes");

// Device address of g_scratch per device, looked up once per device (host code may not
// take the symbol's address itself: on the host, `g_scratch` is only a stand-in).
std::mutex g_scratch_mutex;
double* g_scratch_address[kMaxDevices] = {};

__global__ void __launch_bounds__(kThreads) k_loss_sums_fixed(const float4* __restrict__ pixel_loss, uint64_t pixels,
                                                              double* __restrict__ scratch, double* __restrict__ sums) {
    __shared__ double s[4][kThreads];
    __shared__ bool last;
    double* partials = scratch;
    unsigned int* done = reinterpret_cast<unsigned int*>(scratch + 4 * kMaxBlocks);
    const uint32_t t = threadIdx.x;
    const uint64_t begin = (uint64_t)blockIdx.x * kPixelsPerBlock;
    const uint64_t end = min(begin + kPixelsPerBlock, pixels);
    double a = 0.0, b = 0.0, c = 0.0, d = 0.0;
    for (uint64_t i = begin + t; i < end; i += kThreads) {
        const float4 v = pixel_loss[i];
        a += v.x;
        b += v.y;
        c += v.z;
        d += v.w;
    }
    s[0][t] = a;
    s[1][t] = b;
    s[2][t] = c;
    s[3][t] = d;
    __syncthreads();
    for (int half = kThreads / 2; half > 0; half >>= 1) {
        if (t < (uint32_t)half)
            for (int k = 0; k < 4; ++k) s[k][t] += s[k][t + half];
        __syncthreads();
    }
    if (t < 4) partials[blockIdx.x * 4 + t] = s[t][0];
    __threadfence();
    __syncthreads();
    if (t == 0) last = atomicAdd(done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (t < 4) {
        double sum = 0.0;
        for (uint32_t k = 0; k < gridDim.x; ++k) sum += __ldcg(partials + k * 4 + t);
        sums[t] = sum;
    }
}

// The scratch address on the current device, looked up on the first call on that device.
cudaError_t scratch_address(int device, double** out) {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_address[device]) {
        void* address = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&address, g_scratch);
        if (err != cudaSuccess) return err;
        g_scratch_address[device] = static_cast<double*>(address);
    }
    *out = g_scratch_address[device];
    return cudaSuccess;
}

}  // namespace
}  // namespace splat

extern "C" sp_status sp_loss_sums_noalloc(int device, const float* d_pixel_loss, uint64_t pixel_count, double* d_sums,
                                          void* stream) {
    using namespace splat;
    if (!d_pixel_loss || !d_sums) return SP_ERR_INVALID;
    if (pixel_count == 0 || pixel_count > SP_NOALLOC_MAX_PIXELS) return SP_ERR_INVALID;
    // The kernel reads the pixels as float4 and writes the sums as doubles: a sub-view of a
    // caller's buffer that is not aligned for them is refused here, before anything runs,
    // instead of faulting on the device.
    if ((reinterpret_cast<uintptr_t>(d_pixel_loss) & 15u) != 0 || (reinterpret_cast<uintptr_t>(d_sums) & 7u) != 0)
        return SP_ERR_INVALID;
    if (device < 0 || device >= kMaxDevices) return SP_ERR_INVALID;
    int previous = 0;
    if (cudaGetDevice(&previous) != cudaSuccess) return SP_ERR_CUDA;
    if (previous != device && cudaSetDevice(device) != cudaSuccess) return SP_ERR_CUDA;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    double* scratch = nullptr;
    cudaError_t err = scratch_address(device, &scratch);
    if (err == cudaSuccess)
        err = cudaMemsetAsync(scratch + 4 * kMaxBlocks, 0, sizeof(double), st);
    if (err == cudaSuccess) {
        const unsigned blocks = (unsigned)((pixel_count + kPixelsPerBlock - 1) / kPixelsPerBlock);
        k_loss_sums_fixed<<<blocks, kThreads, 0, st>>>(reinterpret_cast<const float4*>(d_pixel_loss), pixel_count,
                                                        scratch, d_sums);
        err = cudaGetLastError();
    }
    if (previous != device) cudaSetDevice(previous);
    return err == cudaSuccess ? SP_OK : SP_ERR_CUDA;
}
