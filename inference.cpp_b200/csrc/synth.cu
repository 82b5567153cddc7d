// Seeded synthetic weights (see synth.cuh): a host version (threads over
// blocks) and a device version (one thread per block), bit-identical.
// This translation unit is compiled with -fmad=false and the host compiler with
// -ffp-contract=off so neither side fuses multiply-adds.
#include <thread>
#include <vector>

#include "common.cuh"
#include "synth.cuh"

namespace ib {

__global__ void synth_kernel(int type, uint64_t seed, float stdv, int64_t cols, int64_t n_blocks,
                             uint8_t* out) {
    const int bb = ib_synth::block_bytes(type);
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < n_blocks;
         b += (int64_t)gridDim.x * blockDim.x) {
        uint8_t blk[256];
        ib_synth::encode_block(type, seed, stdv, cols, b, blk);
        uint8_t* o = out + b * bb;
        for (int i = 0; i < bb; ++i) o[i] = blk[i];
    }
}

__global__ void synth_f32_kernel(uint64_t seed, float stdv, int64_t n, float* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = ib_synth::value(seed, (uint64_t)i, stdv);
}

}  // namespace ib

using namespace ib;

static int synth_check(int type, int64_t rows, int64_t cols) {
    IB_REQUIRE(rows >= 0 && cols >= 0, "negative shape");
    if (type == IB_TYPE_F32) return IB_OK;
    if (!is_quant(type)) {
        set_error("synth: unsupported type");
        return IB_ERR_UNSUPPORTED;
    }
    IB_REQUIRE(cols % block_elems(type) == 0, "cols must be a multiple of the block size");
    return IB_OK;
}

extern "C" int ib_synth_host(int type, int64_t rows, int64_t cols, uint64_t seed, float stdv,
                             void* host_out, int n_threads) {
    int st = synth_check(type, rows, cols);
    if (st != IB_OK) return st;
    IB_REQUIRE(host_out != nullptr, "null output");
    if (n_threads <= 0) n_threads = (int)std::thread::hardware_concurrency();
    if (n_threads <= 0) n_threads = 1;
    if (type == IB_TYPE_F32) return ib_synth_values_host(rows * cols, seed, stdv, (float*)host_out);
    const int64_t nb = rows * (cols / block_elems(type));
    const int bb = block_bytes(type);
    uint8_t* out = (uint8_t*)host_out;
    auto work = [&](int64_t b0, int64_t b1) {
        for (int64_t b = b0; b < b1; ++b) ib_synth::encode_block(type, seed, stdv, cols, b, out + b * bb);
    };
    if (n_threads == 1 || nb < 4096) {
        work(0, nb);
        return IB_OK;
    }
    std::vector<std::thread> th;
    const int64_t per = (nb + n_threads - 1) / n_threads;
    for (int t = 0; t < n_threads; ++t) {
        const int64_t b0 = t * per, b1 = b0 + per < nb ? b0 + per : nb;
        if (b0 >= b1) break;
        th.emplace_back(work, b0, b1);
    }
    for (auto& t : th) t.join();
    return IB_OK;
}

extern "C" int ib_synth_values_host(int64_t n, uint64_t seed, float stdv, float* host_out) {
    IB_REQUIRE(n >= 0 && host_out, "bad arguments");
    for (int64_t i = 0; i < n; ++i) host_out[i] = ib_synth::value(seed, (uint64_t)i, stdv);
    return IB_OK;
}

extern "C" int ib_synth_device(int type, int64_t rows, int64_t cols, uint64_t seed, float stdv,
                               void* dev_out, void* stream) {
    int st = synth_check(type, rows, cols);
    if (st != IB_OK) return st;
    IB_REQUIRE(dev_out != nullptr, "null output");
    if (rows * cols == 0) return IB_OK;
    if (type == IB_TYPE_F32) {
        synth_f32_kernel<<<148 * 16, 256, 0, as_stream(stream)>>>(seed, stdv, rows * cols,
                                                                 (float*)dev_out);
        IB_LAUNCH_CHECK("synth_f32_kernel");
        return IB_OK;
    }
    const int64_t nb = rows * (cols / block_elems(type));
    int64_t grid = (nb + 127) / 128;
    if (grid > 148 * 64) grid = 148 * 64;
    synth_kernel<<<(unsigned)grid, 128, 0, as_stream(stream)>>>(type, seed, stdv, cols, nb,
                                                                (uint8_t*)dev_out);
    IB_LAUNCH_CHECK("synth_kernel");
    return IB_OK;
}
