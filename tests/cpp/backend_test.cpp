// The reference's CudaTest cases (tests/test_tensor.cpp:337-580) written against
// the inference::cuda mirror in include/ib_cuda_backend.hpp, plus the quantized
// entry points.  Each case compares the device result with a double-precision
// host loop.  Exit status 0 = all passed, 77 = no CUDA device, 1 = failure.
//
//   g++ -std=c++17 -I include tests/cpp/backend_test.cpp -L inference.cpp_b200
//       -lib_cuda -Wl,-rpath,inference.cpp_b200
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "ib_cuda.h"
#include "ib_cuda_backend.hpp"

using namespace inference::cuda;

namespace {

int g_fail = 0;

// |got - want| <= tol * (1 + mag), mag = sum of |terms| when given, else |want|
bool close_all(const std::vector<float>& got, const std::vector<double>& want, double tol,
               const char* what, const std::vector<double>* mag = nullptr) {
    for (size_t i = 0; i < want.size(); ++i) {
        double d = std::fabs((double)got[i] - want[i]);
        double m = mag ? (*mag)[i] : std::fabs(want[i]);
        if (!(d <= tol * (1.0 + m))) {
            std::printf("  %s[%zu]: got %.8g want %.8g\n", what, i, got[i], want[i]);
            return false;
        }
    }
    return true;
}

std::vector<float> randv(size_t n, uint32_t seed, float lo = -1.f, float hi = 1.f) {
    std::mt19937 g(seed);
    std::uniform_real_distribution<float> u(lo, hi);
    std::vector<float> v(n);
    for (auto& x : v) x = u(g);
    return v;
}

Buffer put(const std::vector<float>& v) {
    Buffer b = alloc(v.size() * sizeof(float));
    upload(b, v.data(), v.size() * sizeof(float));
    return b;
}

template <typename T>
Buffer put_raw(const std::vector<T>& v) {
    Buffer b = alloc(v.size() * sizeof(T));
    upload(b, v.data(), v.size() * sizeof(T));
    return b;
}

std::vector<float> get(const Buffer& b, size_t n) {
    std::vector<float> v(n);
    download(v.data(), b, n * sizeof(float));
    return v;
}

void run(const char* name, const std::function<bool()>& fn) {
    bool ok = false;
    try {
        ok = fn();
    } catch (const std::exception& e) {
        std::printf("  exception: %s\n", e.what());
    }
    std::printf("[%s] %s\n", ok ? "PASS" : "FAIL", name);
    if (!ok) ++g_fail;
}

// out[h*hd + d] for one query position attending to positions [0, n_pos)
void attention_host(const std::vector<float>& q, const std::vector<float>& kc,
                    const std::vector<float>& vc, int H, int KV, int hd, int max_seq, int n_pos,
                    double scale, double* out) {
    int G = H / KV;
    for (int h = 0; h < H; ++h) {
        int kh = h / G;
        std::vector<double> s(n_pos);
        double m = -1e300;
        for (int p = 0; p < n_pos; ++p) {
            double acc = 0;
            for (int d = 0; d < hd; ++d)
                acc += (double)q[h * hd + d] * kc[((size_t)kh * max_seq + p) * hd + d];
            s[p] = acc * scale;
            m = std::max(m, s[p]);
        }
        double l = 0;
        for (int p = 0; p < n_pos; ++p) l += (s[p] = std::exp(s[p] - m));
        for (int d = 0; d < hd; ++d) {
            double acc = 0;
            for (int p = 0; p < n_pos; ++p) acc += s[p] * vc[((size_t)kh * max_seq + p) * hd + d];
            out[h * hd + d] = acc / l;
        }
    }
}

}  // namespace

int main() {
    if (!available()) {
        std::printf("no CUDA device\n");
        return 77;
    }
    std::printf("device: %s, %zu MiB total\n", device_name().c_str(), total_memory() >> 20);

    run("GemvSmall", [] {
        const int M = 37, N = 300;
        auto W = randv((size_t)M * N, 1), x = randv(N, 2);
        Buffer dW = put(W), dx = put(x), dy = alloc(M * sizeof(float));
        gemv(dW, dx, dy, M, N);
        sync();
        std::vector<double> want(M), mag(M);
        for (int i = 0; i < M; ++i)
            for (int k = 0; k < N; ++k) {
                want[i] += (double)W[(size_t)i * N + k] * x[k];
                mag[i] += std::fabs((double)W[(size_t)i * N + k] * x[k]);
            }
        bool ok = close_all(get(dy, M), want, 1e-5, "y", &mag);
        release(dW), release(dx), release(dy);
        return ok;
    });

    run("RmsNormSmall", [] {
        const int rows = 3, D = 200;
        auto x = randv((size_t)rows * D, 3), w = randv(D, 4, 0.5f, 1.5f);
        Buffer dx = put(x), dw = put(w), dout = alloc(x.size() * sizeof(float));
        rmsnorm(dx, dw, dout, rows, D, 1e-5f);
        sync();
        std::vector<double> want(x.size());
        for (int r = 0; r < rows; ++r) {
            double ss = 0;
            for (int d = 0; d < D; ++d) ss += (double)x[r * D + d] * x[r * D + d];
            double inv = 1.0 / std::sqrt(ss / D + 1e-5);
            for (int d = 0; d < D; ++d) want[r * D + d] = x[r * D + d] * inv * w[d];
        }
        bool ok = close_all(get(dout, x.size()), want, 1e-5, "out");
        release(dx), release(dw), release(dout);
        return ok;
    });

    run("AttentionLongGQA", [] {
        const int H = 8, KV = 2, hd = 64, S = 512, pos = 400;
        auto q = randv((size_t)H * hd, 5), kc = randv((size_t)KV * S * hd, 6),
             vc = randv((size_t)KV * S * hd, 7);
        Buffer dq = put(q), dk = put(kc), dv = put(vc), dout = alloc((size_t)H * hd * 4);
        float scale = 1.f / std::sqrt((float)hd);
        attention(dq, dk, dv, dout, H, KV, hd, S, pos, scale);
        sync();
        std::vector<double> want((size_t)H * hd);
        attention_host(q, kc, vc, H, KV, hd, S, pos + 1, scale, want.data());
        bool ok = close_all(get(dout, want.size()), want, 1e-4, "out");
        release(dq), release(dk), release(dv), release(dout);
        return ok;
    });

    run("GemvInt16", [] {
        const int M = 19, N = 96;
        std::mt19937 g(8);
        std::vector<int16_t> W((size_t)M * N);
        for (auto& v : W) v = (int16_t)((int)(g() % 65535) - 32767);
        auto sc = randv(M, 9, 1e-5f, 1e-4f), x = randv(N, 10);
        Buffer dW = put_raw(W), ds = put(sc), dx = put(x), dy = alloc(M * 4);
        gemv_i16(dW, ds, dx, dy, M, N);
        sync();
        std::vector<double> want(M), mag(M);
        for (int i = 0; i < M; ++i) {
            for (int k = 0; k < N; ++k) {
                want[i] += (double)W[(size_t)i * N + k] * x[k];
                mag[i] += std::fabs((double)W[(size_t)i * N + k] * x[k]);
            }
            want[i] *= sc[i];
            mag[i] *= sc[i];
        }
        bool ok = close_all(get(dy, M), want, 1e-5, "y", &mag);
        release(dW), release(ds), release(dx), release(dy);
        return ok;
    });

    run("GemmInt16Batch", [] {
        const int T = 5, M = 33, K = 64;
        std::mt19937 g(11);
        std::vector<int16_t> W((size_t)M * K);
        for (auto& v : W) v = (int16_t)((int)(g() % 65535) - 32767);
        auto sc = randv(M, 12, 1e-5f, 1e-4f), X = randv((size_t)T * K, 13);
        Buffer dW = put_raw(W), ds = put(sc), dX = put(X), dY = alloc((size_t)T * M * 4);
        gemm_i16(dW, ds, dX, dY, T, M, K);
        sync();
        std::vector<double> want((size_t)T * M), mag((size_t)T * M);
        for (int t = 0; t < T; ++t)
            for (int i = 0; i < M; ++i) {
                double a = 0, b = 0;
                for (int k = 0; k < K; ++k) {
                    double p = (double)W[(size_t)i * K + k] * X[(size_t)t * K + k];
                    a += p;
                    b += std::fabs(p);
                }
                want[(size_t)t * M + i] = a * sc[i];
                mag[(size_t)t * M + i] = b * sc[i];
            }
        bool ok = close_all(get(dY, want.size()), want, 1e-5, "Y", &mag);
        release(dW), release(ds), release(dX), release(dY);
        return ok;
    });

    run("AttentionBatch", [] {
        const int H = 4, KV = 2, hd = 32, S = 64, start = 7, T = 6;
        auto kc = randv((size_t)KV * S * hd, 14), vc = randv((size_t)KV * S * hd, 15),
             q = randv((size_t)T * H * hd, 16);
        Buffer dq = put(q), dk = put(kc), dv = put(vc), dout = alloc(q.size() * 4);
        float scale = 1.f / std::sqrt((float)hd);
        attention_batch(dq, dk, dv, dout, H, KV, hd, S, start, T, scale);
        sync();
        std::vector<double> want(q.size());
        for (int t = 0; t < T; ++t) {
            std::vector<float> qt(q.begin() + (size_t)t * H * hd, q.begin() + (size_t)(t + 1) * H * hd);
            attention_host(qt, kc, vc, H, KV, hd, S, start + t + 1, scale,
                           want.data() + (size_t)t * H * hd);
        }
        bool ok = close_all(get(dout, want.size()), want, 1e-4, "out");
        release(dq), release(dk), release(dv), release(dout);
        return ok;
    });

    run("EmbeddingInt16", [] {
        const int V = 10, D = 48, id = 7;
        std::mt19937 g(17);
        std::vector<int16_t> tab((size_t)V * D);
        for (auto& v : tab) v = (int16_t)((int)(g() % 65535) - 32767);
        auto sc = randv(V, 18, 1e-5f, 1e-4f);
        Buffer dt = put_raw(tab), ds = put(sc), dout = alloc(D * 4);
        embedding_i16(dt, ds, id, dout, D);
        sync();
        std::vector<double> want(D);
        for (int d = 0; d < D; ++d) want[d] = (double)tab[(size_t)id * D + d] * sc[id];
        bool ok = close_all(get(dout, D), want, 1e-6, "out");
        release(dt), release(ds), release(dout);
        return ok;
    });

    run("GemvQ4K", [] {
        const int64_t M = 64, N = 512;
        int64_t nb = 0;
        size_t bytes = 0;
        int64_t be = 0, bb = 0;
        if (ib_type_info(IB_TYPE_Q4_K, &be, &bb) != IB_OK) return false;
        nb = N / be;
        bytes = (size_t)(M * nb * bb);
        std::vector<uint8_t> W(bytes);
        if (ib_synth_host(IB_TYPE_Q4_K, M, N, 19, 0.02f, W.data(), 1) != IB_OK) return false;
        auto x = randv(N, 20);
        Buffer dW = put_raw(W), dx = put(x), dy = alloc(M * 4), dd = alloc((size_t)M * N * 4);
        gemv_q(IB_TYPE_Q4_K, dW, dx, dy, M, N);
        dequantize(IB_TYPE_Q4_K, dW, dd, M, N);
        sync();
        std::vector<float> deq = get(dd, (size_t)M * N);
        std::vector<double> want(M);
        double bound = 0;
        for (int64_t i = 0; i < M; ++i) {
            double a = 0, s = 0;
            for (int64_t k = 0; k < N; ++k) {
                a += (double)deq[i * N + k] * x[k];
                s += std::fabs((double)deq[i * N + k] * x[k]);
            }
            want[i] = a;
            bound = std::max(bound, s);
        }
        std::vector<float> y = get(dy, M);
        bool ok = true;
        for (int64_t i = 0; i < M; ++i)
            if (std::fabs(y[i] - want[i]) > 2e-5 * bound) {
                std::printf("  y[%ld]: got %.8g want %.8g\n", (long)i, y[i], want[i]);
                ok = false;
                break;
            }
        release(dW), release(dx), release(dy), release(dd);
        return ok;
    });

    run("ErrorsThrowRuntimeError", [] {
        Buffer none;
        try {
            gemv(none, none, none, 4, 4);
        } catch (const std::runtime_error& e) {
            return std::strlen(e.what()) > 0;
        }
        return false;
    });

    std::printf("%d failed\n", g_fail);
    return g_fail ? 1 : 0;
}
