// Lifecycle, memory and error entry points of the C ABI.  Replaces the
// reference's driver singleton (src/ops/cuda_backend.cpp:100-162: dlopen,
// cuInit, cuCtxCreate, cuModuleLoadData) with the CUDA runtime: kernels are
// linked into this library for sm_100a, the primary context is used, and the
// current device is selected with ib_init.
#include <mutex>

#include "common.cuh"
#include "decode.cuh"
#include "step.cuh"
#include "gemv_mma.cuh"
#include "ops.cuh"

namespace ib {

static thread_local std::string t_err;

void set_error(const std::string& msg) { t_err = msg; }
const std::string& last_error() { return t_err; }

}  // namespace ib

using namespace ib;

extern "C" const char* ib_last_error(void) { return t_err.c_str(); }

extern "C" int ib_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" int ib_type_info(int type, int64_t* be, int64_t* bb) {
    IB_REQUIRE(be && bb, "null pointer argument");
    if (block_elems(type) == 0) {
        set_error(std::string("unsupported tensor type ") + std::to_string(type));
        return IB_ERR_UNSUPPORTED;
    }
    *be = block_elems(type);
    *bb = block_bytes(type);
    return IB_OK;
}

extern "C" int ib_init(int device) {
    int n = 0;
    IB_CUDA_CHECK(cudaGetDeviceCount(&n));
    IB_REQUIRE(device >= 0 && device < n, "device index out of range");
    cudaDeviceProp prop;
    IB_CUDA_CHECK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) {
        set_error(std::string("CUDA: device ") + prop.name + " is not sm_100 (the library is compiled for sm_100a)");
        return IB_ERR_UNSUPPORTED;
    }
    IB_CUDA_CHECK(cudaSetDevice(device));
    IB_CUDA_CHECK(cudaFree(nullptr));  // create the primary context now
    return IB_OK;
}

extern "C" int ib_available(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return 0;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return 0;
    return prop.major == 10 ? 1 : 0;
}

extern "C" int ib_device_name(char* buf, size_t len) {
    IB_REQUIRE(buf && len > 0, "null buffer");
    int dev = 0;
    IB_CUDA_CHECK(cudaGetDevice(&dev));
    cudaDeviceProp prop;
    IB_CUDA_CHECK(cudaGetDeviceProperties(&prop, dev));
    snprintf(buf, len, "%s", prop.name);
    return IB_OK;
}

extern "C" int ib_memory_info(size_t* free_bytes, size_t* total_bytes) {
    IB_REQUIRE(free_bytes && total_bytes, "null pointer argument");
    IB_CUDA_CHECK(cudaMemGetInfo(free_bytes, total_bytes));
    return IB_OK;
}

extern "C" int ib_sync(void) {
    IB_CUDA_CHECK(cudaDeviceSynchronize());
    return IB_OK;
}

extern "C" int ib_shutdown(void) { return IB_OK; }

extern "C" int ib_alloc(void** dev, size_t bytes) {
    IB_REQUIRE(dev != nullptr, "null pointer argument");
    *dev = nullptr;
    if (bytes == 0) return IB_OK;
    cudaError_t e = cudaMalloc(dev, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error(std::string("CUDA: cuMemAlloc failed: ") + cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? IB_ERR_OOM : IB_ERR_CUDA;
    }
    return IB_OK;
}

extern "C" int ib_free(void* dev) {
    if (!dev) return IB_OK;
    IB_CUDA_CHECK(cudaFree(dev));
    return IB_OK;
}

extern "C" int ib_upload(void* dev, const void* host, size_t bytes, void* stream) {
    if (bytes == 0) return IB_OK;
    IB_REQUIRE(dev && host, "null pointer argument");
    if (stream) {
        IB_CUDA_CHECK(cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, as_stream(stream)));
    } else {
        IB_CUDA_CHECK(cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice));
    }
    return IB_OK;
}

extern "C" int ib_download(void* host, const void* dev, size_t bytes, void* stream) {
    if (bytes == 0) return IB_OK;
    IB_REQUIRE(dev && host, "null pointer argument");
    if (stream) {
        IB_CUDA_CHECK(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, as_stream(stream)));
    } else {
        IB_CUDA_CHECK(cudaMemcpy(host, dev, bytes, cudaMemcpyDeviceToHost));
    }
    return IB_OK;
}

extern "C" int ib_memset(void* dev, int value, size_t bytes, void* stream) {
    if (bytes == 0) return IB_OK;
    IB_REQUIRE(dev, "null pointer argument");
    IB_CUDA_CHECK(cudaMemsetAsync(dev, value, bytes, as_stream(stream)));
    return IB_OK;
}

extern "C" int ib_check_fault(int* code) {
    IB_REQUIRE(code, "null pointer argument");
    int c2 = 0;
    int st = gemv_fault_take(code);
    if (st != IB_OK) return st;
    if ((st = decode_fault_take(&c2)) != IB_OK) return st;
    if (!*code) *code = c2;
    if ((st = gemm_fault_take(&c2)) != IB_OK) return st;
    if (!*code) *code = c2;
    if ((st = gemm_planes_fault_take(&c2)) != IB_OK) return st;
    if (!*code) *code = c2;
    if ((st = step_fault_take(&c2)) != IB_OK) return st;
    if (!*code) *code = c2;
    if (*code) {
        set_error("CUDA: a pipeline wait expired in a GEMV kernel (code " + std::to_string(*code) +
                  "); results of the calls since the last check are invalid");
        return IB_ERR_TIMEOUT;
    }
    return IB_OK;
}
