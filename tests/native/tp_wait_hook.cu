// Test-only hook (not part of the product; built into tests/native/ by
// oracle/build_ref.py). Runs the tensor-parallel residual kernel of the fused
// peer-store reduction, detail::tp_p2p_residual_kernel, on one GPU with a
// world of two whose second rank never stores anything, so the kernel's
// bounded cross-rank wait runs out; then once more with every arrival in
// place. The waits are bounded (wait_ms); nothing here can hang the GPU.

#include <chrono>
#include <cstdint>
#include <vector>

#include "ops/llama_kernels.cuh"

namespace {
float max_abs_diff(const std::vector<float> &a, const std::vector<float> &b) {
    float m = 0.f;
    for (size_t i = 0; i < a.size(); ++i)
        m = std::max(m, std::fabs(a[i] - b[i]));
    return m;
}
} // namespace

// out[0] error word after the run-out, out[1] arrival counter after it (it must
// keep its value), out[2] wall milliseconds of that launch, out[3] largest
// change of the hidden rows (must be 0), out[4] error word after the complete
// run (0), out[5] its counter after the kernel re-armed it (0), out[6] largest
// error of hidden against the rank-order sum. Returns 0, or -1 on a CUDA error.
extern "C" __attribute__((visibility("default"))) int opw_test_tp_wait(int wait_ms, double *out) {
    using namespace opworks;
    const int world = 2, rows = 3, cols = 256, parity = 1;
    const int64_t slot = static_cast<int64_t>(rows) * cols;
    const unsigned target = static_cast<unsigned>(rows) * (cols / 128) * world;
    float *hidden = nullptr, *recv = nullptr;
    unsigned *cnt = nullptr;
    if (cudaMalloc(&hidden, sizeof(float) * slot) != cudaSuccess ||
        cudaMalloc(&recv, sizeof(float) * 2 * world * slot) != cudaSuccess ||
        cudaMalloc(&cnt, sizeof(unsigned) * 4) != cudaSuccess)
        return -1;
    std::vector<float> h0(slot), r(2 * world * slot);
    for (int64_t i = 0; i < slot; ++i)
        h0[i] = 0.25f * static_cast<float>(i % 97) - 3.f;
    for (size_t i = 0; i < r.size(); ++i)
        r[i] = 0.5f * static_cast<float>(i % 13) - 2.f;
    cudaMemcpy(hidden, h0.data(), sizeof(float) * slot, cudaMemcpyHostToDevice);
    cudaMemcpy(recv, r.data(), sizeof(float) * r.size(), cudaMemcpyHostToDevice);
    int *err = sm100::device_error_word();
    cudaMemset(err, 0, sizeof(int));
    const unsigned partial[4] = {0u, 5u, 0u, 0u}; // [2] arrivals | [2] done; 5 < target
    cudaMemcpy(cnt, partial, sizeof(partial), cudaMemcpyHostToDevice);
    const unsigned long long limit = static_cast<unsigned long long>(wait_ms) * 1000000ull;

    auto t0 = std::chrono::steady_clock::now();
    detail::tp_p2p_residual_kernel<<<rows, 128>>>(hidden, recv, cnt, cnt + 2, parity, world, slot, rows, cols, nullptr,
                                                  detail::ActOut{}, detail::RowSumSq{}, err, limit);
    if (cudaDeviceSynchronize() != cudaSuccess)
        return -1;
    out[2] = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    int e = 0;
    unsigned c[4];
    std::vector<float> h(slot);
    cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost);
    cudaMemcpy(c, cnt, sizeof(c), cudaMemcpyDeviceToHost);
    cudaMemcpy(h.data(), hidden, sizeof(float) * slot, cudaMemcpyDeviceToHost);
    out[0] = e;
    out[1] = c[parity];
    out[3] = max_abs_diff(h, h0);

    // every arrival in place: the sum runs and the counter is re-armed
    cudaMemset(err, 0, sizeof(int));
    const unsigned full[4] = {0u, target, 0u, 0u};
    cudaMemcpy(cnt, full, sizeof(full), cudaMemcpyHostToDevice);
    detail::tp_p2p_residual_kernel<<<rows, 128>>>(hidden, recv, cnt, cnt + 2, parity, world, slot, rows, cols, nullptr,
                                                  detail::ActOut{}, detail::RowSumSq{}, err, limit);
    if (cudaDeviceSynchronize() != cudaSuccess)
        return -1;
    cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost);
    cudaMemcpy(c, cnt, sizeof(c), cudaMemcpyDeviceToHost);
    cudaMemcpy(h.data(), hidden, sizeof(float) * slot, cudaMemcpyDeviceToHost);
    std::vector<float> want(h0);
    for (int64_t i = 0; i < slot; ++i) {
        float y = 0.f;
        for (int k = 0; k < world; ++k)
            y += r[(static_cast<int64_t>(parity) * world + k) * slot + i];
        want[i] += y;
    }
    out[4] = e;
    out[5] = c[parity];
    out[6] = max_abs_diff(h, want);
    cudaFree(hidden);
    cudaFree(recv);
    cudaFree(cnt);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
