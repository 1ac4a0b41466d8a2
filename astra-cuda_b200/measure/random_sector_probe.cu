// Random-sector probe: what this B200 delivers for the access pattern of the
// matching step -- single 4-byte accesses at scattered addresses, each one a
// separate 32-byte DRAM sector -- as opposed to the streamed copy bandwidth
// the HBM roofline is quoted against.  Measurement only (bench.py
// --sector-probe); not part of the matching path.
//
// Every thread walks its own chain over a buffer much larger than L2:
//  * "load"  -- dependent loads: the next address depends on the loaded value
//               (the match loop's pointer chase);
//  * "store" -- independent stores to scattered sectors (fill and insert writes);
//  * "rmw"   -- a load then a store of the same word (size updates);
//  * "red"   -- fire-and-forget reductions (portfolio updates);
//  * "store32" -- independent 32-byte stores that cover a whole sector (fill
//               records and 32-byte order slots): L2 needs nothing from DRAM.
// All addresses are sector-aligned and uniformly spread; the result is
// accesses per second for the whole grid, timed with CUDA events.
#include <cuda_runtime.h>

#include <cstdint>

namespace {

__device__ __forceinline__ uint64_t mix(uint64_t x) {  // SplitMix64 output function
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

template <int kMode>
__global__ void __launch_bounds__(256) probe_kernel(uint32_t* buf, uint64_t sectors, int steps,
                                                    uint32_t* sink) {
  const uint64_t tid = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  uint64_t x = mix(tid + 1);
  uint32_t acc = 0;
  for (int s = 0; s < steps; ++s) {
    const uint64_t i = (mix(x) % sectors) * 8;  // first word of a 32-byte sector
    if (kMode == 0) {  // dependent load
      const uint32_t v = __ldcg(buf + i);
      x += v + 1;
      acc += v;
    } else if (kMode == 1) {  // independent store
      __stcg(buf + i, (uint32_t)x);
      x += 1;
    } else if (kMode == 2) {  // load, then store the same word
      const uint32_t v = __ldcg(buf + i);
      __stcg(buf + i, v + 1);
      x += v + 1;
    } else if (kMode == 3) {  // reduction, no return value
      atomicAdd(buf + i, 1u);
      x += 1;
    } else {  // a whole sector in one 256-bit store
      const uint32_t v = (uint32_t)x;
      asm volatile("st.global.cg.v8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" :: "l"(buf + i), "r"(v)
                   : "memory");
      x += 1;
    }
  }
  if (acc == 0xFFFFFFFFu) sink[0] = acc;  // keeps the loads
}

}  // namespace

extern "C" {

// Runs mode 0..4 (load, store, rmw, red, store32) over `bytes` of device memory with
// `blocks` x 256 threads and `steps` accesses per thread; returns the kernel's
// time in milliseconds (median of `reps`), or a negative value on error.
float probe_run(int mode, uint64_t bytes, int blocks, int steps, int reps) {
  uint32_t* buf = nullptr;
  uint32_t* sink = nullptr;
  if (cudaMalloc(&buf, bytes) != cudaSuccess) return -1.f;
  if (cudaMalloc(&sink, 4) != cudaSuccess) { cudaFree(buf); return -1.f; }
  cudaMemset(buf, 0, bytes);
  const uint64_t sectors = bytes / 32;
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  float times[32];
  if (reps > 32) reps = 32;
  for (int r = -1; r < reps; ++r) {  // r = -1 warms up
    cudaEventRecord(a);
    switch (mode) {
      case 0: probe_kernel<0><<<blocks, 256>>>(buf, sectors, steps, sink); break;
      case 1: probe_kernel<1><<<blocks, 256>>>(buf, sectors, steps, sink); break;
      case 2: probe_kernel<2><<<blocks, 256>>>(buf, sectors, steps, sink); break;
      case 3: probe_kernel<3><<<blocks, 256>>>(buf, sectors, steps, sink); break;
      default: probe_kernel<4><<<blocks, 256>>>(buf, sectors, steps, sink); break;
    }
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    if (r >= 0) cudaEventElapsedTime(&times[r], a, b);
  }
  const bool ok = cudaGetLastError() == cudaSuccess;
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaFree(buf);
  cudaFree(sink);
  if (!ok) return -2.f;
  for (int i = 1; i < reps; ++i)  // insertion sort for the median
    for (int j = i; j > 0 && times[j] < times[j - 1]; --j) {
      const float t = times[j]; times[j] = times[j - 1]; times[j - 1] = t;
    }
  return times[reps / 2];
}

}  // extern "C"
