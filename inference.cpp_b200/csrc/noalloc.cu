// ib_gemv_q_noalloc: the fused dequant-GEMV of ib_gemv_q with its activation-limb
// scratch in a fixed file-scope device array, so a call allocates no device memory.
//
// The array's address is resolved once per device with cudaGetSymbolAddress, with
// that device current, on the first call made on it; later calls reuse it.  The same
// one-time set-up prepares every kernel instance the entry point can launch, for all
// six formats (function attributes, shared-memory opt-in, occupancy, module loading),
// so a later first call of another format does no first-use work either.  The cached
// address belongs to the device's primary context: after cudaDeviceReset, or anything
// else that destroys that context, this entry point must not be called again in the
// process.  The scratch needs no initial value: every byte the GEMV kernel reads is
// first written by the limb kernel of the same call, on the same stream.  Two calls in
// flight on one device at once (different streams or host threads without ordering
// between them) share the array and race.
#include <mutex>
#include <string>

#include "common.cuh"
#include "gemv_mma.cuh"
#include "ib_cuda.h"

namespace ib {
namespace {

constexpr int kMaxCols = IB_NOALLOC_MAX_COLS;
// Limb layout of xlimbs_bytes(kMaxCols): 128 B of limbs per 32 elements, a scale
// and a sum per 32, a sum per 16, each part rounded up to 256 bytes.
constexpr size_t kGroups = kMaxCols / 32;
constexpr size_t kScratchBytes = ((kGroups * 128 + 255) / 256 + (kGroups * 4 + 255) / 256 * 2 +
                                  (kGroups * 8 + 255) / 256) * 256;
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_gemv_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

int scratch_address(void** out) {
    int dev = 0;
    IB_CUDA_CHECK(cudaGetDevice(&dev));
    IB_REQUIRE(dev >= 0 && dev < kMaxDevices, "ib_gemv_q_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_scratch);
        if (e != cudaSuccess || p == nullptr) {
            set_error(std::string("CUDA: cudaGetSymbolAddress(g_gemv_scratch) failed: ") +
                      cudaGetErrorString(e));
            return IB_ERR_CUDA;
        }
        const int r = gemv_mma_prepare_device();
        if (r != IB_OK) return r;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return IB_OK;
}

}  // namespace
}  // namespace ib

using namespace ib;

extern "C" int ib_gemv_q_noalloc(int type, const void* dev_W, const float* dev_x, float* dev_y,
                                 int64_t rows, int64_t cols, void* stream) {
    if (rows == 0) return IB_OK;
    IB_REQUIRE(dev_W && dev_x && dev_y, "null pointer argument");
    IB_REQUIRE(rows > 0 && cols > 0 && rows < (1ll << 31), "bad GEMV shape");
    if (!gemv_mma_supported(type)) {
        set_error(std::string("ib_gemv_q_noalloc: unsupported type ") + type_name(type));
        return IB_ERR_UNSUPPORTED;
    }
    IB_REQUIRE(cols % block_elems(type) == 0, "cols must be a multiple of the block size");
    if (cols > kMaxCols) {
        set_error("ib_gemv_q_noalloc: cols = " + std::to_string(cols) + " exceeds the limit of " +
                  std::to_string(kMaxCols) + " (static scratch of " +
                  std::to_string(kScratchBytes) + " bytes); use ib_gemv_q");
        return IB_ERR_INVALID;
    }
    IB_REQUIRE(((uintptr_t)dev_x & 15) == 0, "x must be 16-byte aligned");
    if (((uintptr_t)dev_W % gemv_mma_align(type)) != 0) {
        set_error("ib_gemv_q_noalloc: W must be " + std::to_string(gemv_mma_align(type)) +
                  "-byte aligned for " + type_name(type));
        return IB_ERR_INVALID;
    }
    if (xlimbs_bytes((int)cols) > kScratchBytes) {
        set_error("ib_gemv_q_noalloc: scratch layout larger than the static array");
        return IB_ERR_INVALID;
    }
    void* scratch = nullptr;
    int r = scratch_address(&scratch);
    if (r != IB_OK) return r;
    XLimbs xb;
    xlimbs_carve(scratch, (int)cols, xb);
    cudaStream_t st = as_stream(stream);
    if ((r = xq_launch(dev_x, (int)cols, gemv_mma_group(type), xb, st)) != IB_OK) return r;
    return gemv_mma_launch(type, dev_W, xb, dev_y, rows, cols, st);
}
