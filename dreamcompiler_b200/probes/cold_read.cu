// Measurement program (not part of libdgx): the device time of reading a cold
// 16 MiB buffer once per launch, the floor under the int8 layer's weight
// stream (config 5: an N = K = 4096 int8 weight matrix is 16 MiB). It cycles
// 16 buffers (256 MiB, twice the L2) so every launch misses L2, captures 64
// launches in a CUDA graph and reports the best of 5 replays per launch, for
// several grid shapes of a plain 16-byte-load streaming kernel, plus an empty
// kernel for the per-launch floor of a graph.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o cold_read dreamcompiler_b200/probes/cold_read.cu
//   ./cold_read                       # every shape
//   ./cold_read 2048 256 2            # one shape: blocks, threads, loads in flight per thread
#include <cstdlib>
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>

__global__ void empty_kernel(int* out) {
  if (threadIdx.x == 1023) out[0] = 1;
}

template <int UNROLL>
__global__ void __launch_bounds__(512) read_kernel(const uint4* __restrict__ src, size_t n16, unsigned* out) {
  unsigned acc = 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  for (; i + (UNROLL - 1) * stride < n16; i += UNROLL * stride) {
    uint4 v[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) v[u] = __ldcs(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
  }
  for (; i < n16; i += stride) {
    const uint4 v = __ldcs(src + i);
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (acc == 0x12345678u) out[0] = acc;
}

int main(int argc, char** argv) {
  const size_t bytes = 16u << 20, n16 = bytes / 16;
  const int nbuf = 16, iters = 64, reps = 5;
  uint4* bufs[nbuf];
  for (int b = 0; b < nbuf; ++b) {
    cudaMalloc(&bufs[b], bytes);
    cudaMemset(bufs[b], b + 1, bytes);
  }
  unsigned* out;
  cudaMalloc(&out, 64);
  int nsm;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, 0);
  cudaStream_t s;
  cudaStreamCreate(&s);
  struct Shape { int blocks, threads, unroll; };
  Shape shapes[] = {{0, 0, 0}, {nsm, 512, 8}, {2 * nsm, 512, 4}, {4 * nsm, 256, 4}, {4 * nsm, 512, 2},
                    {8 * nsm, 256, 2}, {16 * nsm, 256, 1}, {2048, 256, 2}};
  const bool one = argc == 4;
  const Shape chosen{one ? atoi(argv[1]) : 0, one ? atoi(argv[2]) : 0, one ? atoi(argv[3]) : 0};
  if (one && (chosen.blocks < 1 || chosen.threads < 32 || chosen.threads > 512 ||
              (chosen.unroll != 1 && chosen.unroll != 2 && chosen.unroll != 4 && chosen.unroll != 8))) {
    printf("usage: cold_read [blocks threads(32..512) unroll(1|2|4|8)]\n");
    return 2;
  }
  for (const Shape& sh : shapes) {
    if (one && &sh != &shapes[0]) break;
    const Shape& use = one ? chosen : sh;
    cudaGraph_t g;
    cudaGraphExec_t ge;
    cudaStreamBeginCapture(s, cudaStreamCaptureModeGlobal);
    for (int i = 0; i < iters; ++i) {
      const uint4* src = bufs[i % nbuf];
      if (use.blocks == 0) empty_kernel<<<1, 32, 0, s>>>((int*)out);
      else if (use.unroll == 8) read_kernel<8><<<use.blocks, use.threads, 0, s>>>(src, n16, out);
      else if (use.unroll == 4) read_kernel<4><<<use.blocks, use.threads, 0, s>>>(src, n16, out);
      else if (use.unroll == 2) read_kernel<2><<<use.blocks, use.threads, 0, s>>>(src, n16, out);
      else read_kernel<1><<<use.blocks, use.threads, 0, s>>>(src, n16, out);
    }
    cudaStreamEndCapture(s, &g);
    cudaGraphInstantiate(&ge, g, 0);
    cudaGraphLaunch(ge, s);
    cudaStreamSynchronize(s);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    float best = 1e9;
    for (int r = 0; r < reps; ++r) {
      cudaEventRecord(e0, s);
      cudaGraphLaunch(ge, s);
      cudaEventRecord(e1, s);
      cudaStreamSynchronize(s);
      float ms;
      cudaEventElapsedTime(&ms, e0, e1);
      if (ms < best) best = ms;
    }
    const double us = best * 1e3 / iters;
    if (use.blocks == 0)
      printf("empty kernel: %.2f us per launch\n", us);
    else
      printf("read 16 MiB cold: grid %d x %d unroll %d: %.2f us per launch = %.0f GB/s\n", use.blocks, use.threads,
             use.unroll, us, bytes / us / 1e3);
    cudaGraphExecDestroy(ge);
    cudaGraphDestroy(g);
  }
  cudaError_t e = cudaDeviceSynchronize();
  printf("status %s\n", cudaGetErrorString(e));
  return e == cudaSuccess ? 0 : 1;
}
