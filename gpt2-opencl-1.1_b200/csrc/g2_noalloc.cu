// g2_noalloc.cu -- g2k_matvec_noalloc: the split-K GEMV of g2k_matvec with its
// scratch in a fixed device array, for callers that cannot allocate device
// memory.
//
// Who needs it: a host that drives single kernels through this C ABI but has
// no device allocator of its own to hand it a workspace -- a cgo / JNI / FFI
// binding, or an application whose device memory is fully owned by another
// allocator -- and code on a latency-critical path where cudaMalloc's implicit
// device synchronisation is not acceptable.  Those callers still pass the
// inputs and outputs; the scratch comes from here.
//
// The scratch is one file-scope __device__ array of kNoallocScratchBytes
// (256 KiB), present on every GPU that loads this library until the process
// exits.  Host code cannot use the array's name as a device address, so the
// first call on each device, with that device current, looks the address up
// with cudaGetSymbolAddress and caches it; make that first call on a device
// before any stream capture.  The cached address belongs to the device's
// current context: after cudaDeviceReset on a device the library's module is
// loaded afresh at another address, so do not call this entry point again on
// that device in the same process.  All calls share the array: each call clears the
// split-K counters (cudaMemsetAsync, no allocation) before its kernel, and
// calls that overlap on the GPU (concurrent streams, or several host
// threads) race on the array and must be serialised by the caller.
#include <mutex>

#include "g2_internal.h"
#include "gpt2b200.h"

namespace {

constexpr size_t kNoallocScratchBytes = 256 * 1024;
static __device__ __align__(256) unsigned char g_matvec_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_dev[kMaxDevices];   // device address of g_matvec_scratch per device

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

extern "C" int g2k_matvec_noalloc(const float *x, const float *W, const float *bias, const float *residual, float *y,
                                  int N, int K, int apply_gelu, const float *ln_gamma, const float *ln_beta,
                                  void *stream) {
    if (!x || !W || !y) return g2::set_error(G2_ERR_ARG, "g2k_matvec_noalloc: null argument");
    if (N <= 0 || K <= 0 || N % 4 || K % 16)
        return g2::set_error(G2_ERR_ARG, "g2k_matvec_noalloc: need N % 4 == 0 and K % 16 == 0");
    if ((ln_gamma == nullptr) != (ln_beta == nullptr))
        return g2::set_error(G2_ERR_ARG, "g2k_matvec_noalloc: ln_gamma and ln_beta go together");
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return g2::set_error(G2_ERR_CUDA, "g2k_matvec_noalloc: no current CUDA device");
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return g2::set_error(G2_ERR_CUDA, "g2k_matvec_noalloc: cannot query the device");
    const g2::GemvPlan p = g2::gemv_plan<float>(N, K, sms);
    const size_t ctr_bytes = align256((size_t)p.tiles * sizeof(unsigned));
    const size_t need = ctr_bytes + align256((size_t)p.ksplit * N * sizeof(float));
    if (need > kNoallocScratchBytes)
        return g2::set_error(G2_ERR_RANGE, "g2k_matvec_noalloc: this N x K needs more than the 256 KiB of fixed "
                                           "scratch; use g2k_matvec with a caller-provided workspace");
    if (p.smem_bytes > g2::kGemvMaxSmem)
        return g2::set_error(G2_ERR_RANGE, "g2k_matvec_noalloc: K is too long for one column tile's shared memory "
                                           "at this N");
    // An error left pending by earlier work of the caller is reported as such,
    // not as this call's launch failure.
    if (cudaPeekAtLastError() != cudaSuccess)
        return g2::set_error(G2_ERR_CUDA, "g2k_matvec_noalloc: a CUDA error was already pending before this call");
    void *base;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_scratch_dev[dev]) {
            void *ptr = nullptr;
            if (cudaGetSymbolAddress(&ptr, g_matvec_scratch) != cudaSuccess || !ptr)
                return g2::set_error(G2_ERR_CUDA, "g2k_matvec_noalloc: cudaGetSymbolAddress failed");
            g_scratch_dev[dev] = ptr;
        }
        base = g_scratch_dev[dev];
    }
    cudaStream_t st = (cudaStream_t)stream;
    unsigned *ctr = reinterpret_cast<unsigned *>(base);
    float *partial = reinterpret_cast<float *>((char *)base + ctr_bytes);
    if (cudaMemsetAsync(ctr, 0, ctr_bytes, st) != cudaSuccess)
        return g2::set_error(G2_ERR_CUDA, "g2k_matvec_noalloc: clearing the counters failed");
    const int epi = (bias ? g2::EPI_BIAS : 0) | (apply_gelu ? g2::EPI_GELU : 0) | (residual ? g2::EPI_RESID : 0);
    g2::launch_gemv<float>(x, W, bias, residual, y, N, K, epi, ln_gamma, ln_beta, partial, ctr, p, nullptr, 0, nullptr,
                           nullptr, st);
    if (cudaGetLastError() != cudaSuccess) return g2::set_error(G2_ERR_CUDA, "g2k_matvec_noalloc: launch failed");
    return G2_OK;
}
