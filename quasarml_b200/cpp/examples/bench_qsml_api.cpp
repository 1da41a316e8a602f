// The workloads of the reference's benchmark program
// (unit-tests/src/_bench_qsml_performance.cpp: add/mul on 1M and 10M
// elements, square matmul, activations and softmax on 1M, sum/mean/max on 1M)
// run through this backend's qsml:: API, timed the way that program times
// them: wall clock around the calls, synchronize() before reading the clock.
// It also times host <-> device transfers from ordinary (pageable) memory.
// Numbers are printed only; nothing is checked (the tests do that).
#include <QuasarML.h>

#include <chrono>
#include <cstdio>
#include <vector>

using clk = std::chrono::steady_clock;

template <typename F> static double time_ms(F&& f, int iters) {
    f();  // warm-up
    qsml::synchronize();
    const auto t0 = clk::now();
    for (int i = 0; i < iters; ++i) f();
    qsml::synchronize();
    return std::chrono::duration<double, std::milli>(clk::now() - t0).count() / iters;
}

int main() {
    qsml::init();
    std::printf("device: %s\n", qsml::device_names().empty() ? "?" : qsml::device_names()[0].c_str());

    std::printf("\nelementwise (GFLOP/s, 1 flop per element)\n");
    for (qsml::u32 n : {1u << 20, 10u << 20}) {
        auto a = qsml::ones({n}), b = qsml::ones({n});
        const double add = time_ms([&] { auto c = qsml::add(a, b); }, 100);
        const double mul = time_ms([&] { auto c = qsml::mul(a, b); }, 100);
        std::printf("  n=%-9u add %.3f ms (%.1f GFLOP/s)  mul %.3f ms (%.1f GFLOP/s)\n", n, add, n / add / 1e6, mul,
                    n / mul / 1e6);
    }

    std::printf("\nmatmul fp32, reference fma order (GFLOP/s)\n");
    for (qsml::u32 n : {256u, 512u, 1024u, 2048u, 4096u, 8192u}) {
        auto a = qsml::ones({n, n}), b = qsml::ones({n, n});
        const int iters = n >= 4096 ? 3 : 20;
        const double ms = time_ms([&] { auto c = qsml::matmul(a, b); }, iters);
        std::printf("  %5u^3  %9.3f ms  %10.1f GFLOP/s\n", n, ms, 2.0 * n * n * n / ms / 1e6);
    }
    std::printf("\nmatmul fp16 inputs, fp32 out, tensor cores (GFLOP/s)\n");
    for (qsml::u32 n : {1024u, 4096u, 8192u}) {
        auto a = qsml::ones({n, n}, qsml::DataType::F16), b = qsml::ones({n, n}, qsml::DataType::F16);
        const double ms = time_ms([&] { auto c = qsml::matmul(a, b, qsml::DataType::F32); }, 10);
        std::printf("  %5u^3  %9.3f ms  %10.1f GFLOP/s\n", n, ms, 2.0 * n * n * n / ms / 1e6);
    }

    std::printf("\nactivations on 1M elements (ms/op)\n");
    {
        auto x = qsml::ones({1u << 20});
        std::printf("  relu %.4f  sigmoid %.4f  gelu %.4f  softmax %.4f\n",
                    time_ms([&] { auto y = qsml::relu(x); }, 100), time_ms([&] { auto y = qsml::sigmoid(x); }, 100),
                    time_ms([&] { auto y = qsml::gelu(x); }, 100), time_ms([&] { auto y = qsml::softmax(x); }, 100));
    }

    std::printf("\nreductions on 1M elements (ms/op)\n");
    {
        auto x = qsml::ones({1u << 20});
        std::printf("  sum %.4f  mean %.4f  max %.4f\n", time_ms([&] { auto y = qsml::sum(x); }, 100),
                    time_ms([&] { auto y = qsml::mean(x); }, 100), time_ms([&] { auto y = qsml::max(x); }, 100));
    }

    std::printf("\nhost <-> device from pageable memory, 256 MiB (GB/s)\n");
    {
        const qsml::u32 n = 64u << 20;  // floats
        std::vector<float> h(n, 1.0f);
        auto t = qsml::empty({n});
        const double up = time_ms([&] { t->upload(h.data()); }, 5);
        const double down = time_ms([&] { t->download(h.data()); }, 5);
        std::printf("  upload %.1f GB/s  download %.1f GB/s\n", n * 4.0 / up / 1e6, n * 4.0 / down / 1e6);
    }
    qsml::shutdown();
    return 0;
}
