// Measurement kernel: the FP64 pipe's throughput on this part, timed by the caller with CUDA events. It is the
// denominator of the FP64-pipe fractions the benchmark reports (the NTT passes, base conversion and the inner products
// run their modular products as FP64 FMA pairs), in place of the nominal 64 FMA / clock / SM.
#include "kernels.h"

namespace pcb {
namespace probe {

constexpr int CHAINS = 8;  // independent FMA chains per thread: enough to cover the FMA latency at 32 warps per SM
constexpr int THREADS = 256;

__global__ void __launch_bounds__(THREADS) fma_loop(double* sink, int iters, double a, double b) {
    double x[CHAINS];
#pragma unroll
    for (int c = 0; c < CHAINS; ++c) x[c] = 1e-3 * (threadIdx.x + c);
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int c = 0; c < CHAINS; ++c) x[c] = fma(x[c], a, b);
    }
    double s = 0.0;
#pragma unroll
    for (int c = 0; c < CHAINS; ++c) s += x[c];
    if (s == -1.0) sink[blockIdx.x] = s;  // keeps the chains live; x converges to b / (1 - a) > 0
}

}  // namespace probe
}  // namespace pcb

// Launches iters x 8 FMAs on every thread of 4 x 256-thread blocks per SM; returns the FMA count (or a negative
// cudaError_t). `sink` holds one double per block (never written in practice).
extern "C" int64_t pcb_fp64_fma_loop(double* sink, int32_t iters, cudaStream_t s) {
    int dev = 0, sms = 0;
    if (!sink || iters < 1) return -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return -(int64_t)e;
    const int blocks = 4 * sms;
    pcb::probe::fma_loop<<<blocks, pcb::probe::THREADS, 0, s>>>(sink, iters, 0.999999, 1e-6);
    e = cudaGetLastError();
    if (e != cudaSuccess) return -(int64_t)e;
    return (int64_t)blocks * pcb::probe::THREADS * pcb::probe::CHAINS * iters;
}
