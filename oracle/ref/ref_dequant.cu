// Test infrastructure (pins the oracle; never on the product path).
//
// Host launcher for the reference's own CUDA dequantization kernels, compiled
// from the reference's sources by oracle/ref/Makefile into oracle/_ref/:
// `dequantize_block_q4_K_f32` / `dequantize_block_q6_K_f32`
// (ferrite-os/crates/internal/ptx-kernels/kernels/candle/quantized.cu:936-1022,
// 1024-1129, instantiated at :1130-1151): one CTA per GGUF super-block, 32
// threads for Q4_K and 64 for Q6_K (the launch shapes those kernels assume),
// output y[256 * block + i] f32 in GGUF element order.
#include <cuda_runtime.h>
#include <stdint.h>

extern "C" __global__ void dequantize_block_q4_K_f32(const void *__restrict__ vx, float *__restrict__ y);
extern "C" __global__ void dequantize_block_q6_K_f32(const void *__restrict__ vx, float *__restrict__ y);

// dtype: 12 = Q4_K, 14 = Q6_K (GGML type ids); returns a cudaError_t value.
extern "C" int ref_dequantize_host(int dtype, const void *blocks, int64_t nblocks, float *out) {
    const size_t bb = dtype == 12 ? 144 : 210;
    void *dx = nullptr;
    float *dy = nullptr;
    cudaError_t e = cudaMalloc(&dx, bb * (size_t)nblocks);
    if (e == cudaSuccess) e = cudaMalloc(&dy, 256 * sizeof(float) * (size_t)nblocks);
    if (e == cudaSuccess) e = cudaMemcpy(dx, blocks, bb * (size_t)nblocks, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        if (dtype == 12) dequantize_block_q4_K_f32<<<(unsigned)nblocks, 32>>>(dx, dy);
        else dequantize_block_q6_K_f32<<<(unsigned)nblocks, 64>>>(dx, dy);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(out, dy, 256 * sizeof(float) * (size_t)nblocks, cudaMemcpyDeviceToHost);
    cudaFree(dx);
    cudaFree(dy);
    return (int)e;
}
