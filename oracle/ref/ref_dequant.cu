// Test infrastructure (pins the oracle; never on the product path).
//
// Host launchers for the reference's own CUDA kernels, compiled from the
// reference's sources by oracle/ref/Makefile into oracle/_ref/.  Dequantization:
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

// The reference's decode QMatMul kernels for one activation row, launched
// with the shapes candle's CUDA backend uses for them:
//   mode 0: quantize_q8_1 (quantized.cu:3348; 256-thread blocks, rows padded
//           to 512) then mul_mat_vec_q{4,6}_K_q8_1_cuda1 (:2757, :2773; 4 warps
//           per output row) -- the integer MMVQ path;
//   mode 1: dequantize_mul_mat_vec_q{4,6}_k (:1456, :1708; one warp per
//           output row) -- the float DMMV path.
// w: n rows of k/256 GGUF blocks, x: k f32, y: n f32.  Returns a cudaError_t.
extern "C" __global__ void quantize_q8_1(const float *__restrict__ x, void *__restrict__ vy, const int kx,
                                         const int kx_padded);
extern "C" __global__ void mul_mat_vec_q4_K_q8_1_cuda1(const void *vx, const void *vy, float *dst, const int ncols_x,
                                                       const int nrows_x, const int nrows_y, const int nrows_dst);
extern "C" __global__ void mul_mat_vec_q6_K_q8_1_cuda1(const void *vx, const void *vy, float *dst, const int ncols_x,
                                                       const int nrows_x, const int nrows_y, const int nrows_dst);
extern "C" __global__ void dequantize_mul_mat_vec_q4_k(const void *__restrict__ vx, const float *__restrict__ yy,
                                                       float *__restrict__ dst, const int ncols, int nrows);
extern "C" __global__ void dequantize_mul_mat_vec_q6_k(const void *__restrict__ vx, const float *__restrict__ yy,
                                                       float *__restrict__ dst, const int ncols, int nrows);

extern "C" int ref_qmatmul_vec_host(int dtype, int mode, const void *w, int n, int k, const float *x, float *y) {
    const size_t bb = dtype == 12 ? 144 : 210;
    const size_t wbytes = bb * (size_t)n * (size_t)(k / 256);
    const int kpad = (k + 511) / 512 * 512;
    void *dw = nullptr, *dq = nullptr;
    float *dx = nullptr, *dy = nullptr;
    cudaError_t e = cudaMalloc(&dw, wbytes);
    if (e == cudaSuccess) e = cudaMalloc(&dx, sizeof(float) * (size_t)k);
    if (e == cudaSuccess) e = cudaMalloc(&dy, sizeof(float) * (size_t)n);
    if (e == cudaSuccess) e = cudaMalloc(&dq, (size_t)(kpad / 32) * 36);
    if (e == cudaSuccess) e = cudaMemcpy(dw, w, wbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(dx, x, sizeof(float) * (size_t)k, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        if (mode == 0) {
            quantize_q8_1<<<dim3((unsigned)((kpad + 255) / 256), 1), dim3(256, 1)>>>(dx, dq, k, kpad);
            if (dtype == 12) mul_mat_vec_q4_K_q8_1_cuda1<<<(unsigned)n, dim3(32, 4)>>>(dw, dq, dy, k, n, kpad, n);
            else mul_mat_vec_q6_K_q8_1_cuda1<<<(unsigned)n, dim3(32, 4)>>>(dw, dq, dy, k, n, kpad, n);
        } else {
            if (dtype == 12) dequantize_mul_mat_vec_q4_k<<<(unsigned)n, dim3(32, 1)>>>(dw, dx, dy, k, n);
            else dequantize_mul_mat_vec_q6_k<<<(unsigned)n, dim3(32, 1)>>>(dw, dx, dy, k, n);
        }
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(y, dy, sizeof(float) * (size_t)n, cudaMemcpyDeviceToHost);
    cudaFree(dw);
    cudaFree(dx);
    cudaFree(dy);
    cudaFree(dq);
    return (int)e;
}

// Device time of the reference's integer decode QMatMul (quantize_q8_1 +
// mul_mat_vec_q*_K_q8_1_cuda1, one activation row) averaged over `iters`
// back-to-back launches after `warm` untimed ones; inputs resident on the
// device.  Returns a cudaError_t; *ms_out = milliseconds per QMatMul.
extern "C" int ref_qmatmul_vec_time(int dtype, const void *w, int n, int k, const float *x, int warm, int iters,
                                    float *ms_out) {
    const size_t bb = dtype == 12 ? 144 : 210;
    const size_t wbytes = bb * (size_t)n * (size_t)(k / 256);
    const int kpad = (k + 511) / 512 * 512;
    void *dw = nullptr, *dq = nullptr;
    float *dx = nullptr, *dy = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t e = cudaMalloc(&dw, wbytes);
    if (e == cudaSuccess) e = cudaMalloc(&dx, sizeof(float) * (size_t)k);
    if (e == cudaSuccess) e = cudaMalloc(&dy, sizeof(float) * (size_t)n);
    if (e == cudaSuccess) e = cudaMalloc(&dq, (size_t)(kpad / 32) * 36);
    if (e == cudaSuccess) e = cudaMemcpy(dw, w, wbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(dx, x, sizeof(float) * (size_t)k, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    auto run = [&] {
        quantize_q8_1<<<dim3((unsigned)((kpad + 255) / 256), 1), dim3(256, 1)>>>(dx, dq, k, kpad);
        if (dtype == 12) mul_mat_vec_q4_K_q8_1_cuda1<<<(unsigned)n, dim3(32, 4)>>>(dw, dq, dy, k, n, kpad, n);
        else mul_mat_vec_q6_K_q8_1_cuda1<<<(unsigned)n, dim3(32, 4)>>>(dw, dq, dy, k, n, kpad, n);
    };
    if (e == cudaSuccess) {
        for (int i = 0; i < warm; i++) run();
        cudaEventRecord(e0);
        for (int i = 0; i < iters; i++) run();
        cudaEventRecord(e1);
        e = cudaEventSynchronize(e1);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    *ms_out = iters > 0 ? ms / iters : 0.f;
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(dw);
    cudaFree(dx);
    cudaFree(dy);
    cudaFree(dq);
    return (int)e;
}
