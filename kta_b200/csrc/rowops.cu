// Row-wise RMSNorm and softmax over [M, N] f16/bf16 matrices, sm_100a.
//
//   RMSNorm: Y = X * rsqrt(mean_j(X^2) + eps) * W     (KTA's rmsnorm, perfmodel/testset/gen.py:662-704)
//   softmax: Y = 2^(X log2(e) - max) / sum             (KTA's softmax, perfmodel/testset/gen.py:781-807)
//
// Both read X once and write Y once: HBM-bound at 4 bytes per element (plus W once for RMSNorm,
// which stays in L2). A row belongs to a group of G threads (G = 32..256, a power of two); each
// thread keeps EPT elements of it in registers (16-byte vectors, consecutive threads on
// consecutive vectors, so every warp load is 512 contiguous bytes); the fp32 reductions run
// over warp shuffles and, for G > 32, a small shared-memory exchange between the group's
// warps. A CTA of 256 threads holds 256 / G rows; the grid covers M. Statistics and the
// arithmetic are fp32 as in the reference; the output is rounded once to the storage type.
#include <algorithm>
#include <cmath>
#include <type_traits>

#include "kta_common.cuh"
#include "kta_host.h"

namespace kta {
namespace rowops {

constexpr int THREADS = 256;
constexpr int MAX_EPT = 64;  // elements per thread: N <= 256 * 64 = 16384

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// sum or max over the G threads of a row group (G a power of two, 32 <= G <= 256);
// `red` holds THREADS / 32 floats per CTA
template <int G, bool MAX>
__device__ __forceinline__ float group_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, w) : v + w;
  }
  if constexpr (G > 32) {
    constexpr int W = G / 32;  // warps per row group
    const int warp = threadIdx.x >> 5;
    const int first = warp & ~(W - 1);
    __syncthreads();  // the previous reduction's reads of `red` are done
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    v = red[first];
#pragma unroll
    for (int i = 1; i < W; ++i) v = MAX ? fmaxf(v, red[first + i]) : v + red[first + i];
  }
  return v;
}

// OP 0: RMSNorm, OP 1: softmax. Row r of the grid: CTA blockIdx.x, group threadIdx.x / G.
template <int G, int EPT, typename T, int OP>
__global__ void __launch_bounds__(THREADS)
    rowop_kernel(const T* __restrict__ X, const T* __restrict__ W, T* __restrict__ Y, int M,
                 int N, float eps) {
  __shared__ float red[THREADS / 32];
  pdl_launch_dependents();
  pdl_wait();  // the previous grid's writes (this launch's inputs) are visible from here on
  constexpr int VEC = 8;                 // 16-byte vectors of 16-bit elements
  constexpr int NV = EPT / VEC;          // vectors per thread
  const int g = threadIdx.x % G;
  const long long row = static_cast<long long>(blockIdx.x) * (THREADS / G) + threadIdx.x / G;
  const bool live = row < M;
  const T* xr = X + row * N;
  T* yr = Y + row * N;
  float v[EPT];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * G + g) * VEC;  // first column of this vector
    if (live && c < N) {
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(xr + c));  // read once: streaming
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[i * VEC + k] = to_f<T>(e[k]);
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[i * VEC + k] = OP == 0 ? 0.f : -INFINITY;
    }
  }
  if constexpr (OP == 0) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < EPT; ++k) ss = fmaf(v[k], v[k], ss);
    ss = group_reduce<G, false>(ss, red);
    const float inv = rsqrtf(ss / static_cast<float>(N) + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * G + g) * VEC;
      if (live && c < N) {
        const uint4 wu = __ldg(reinterpret_cast<const uint4*>(W + c));
        const T* we = reinterpret_cast<const T*>(&wu);
        uint4 out;
        T* oe = reinterpret_cast<T*>(&out);
#pragma unroll
        for (int k = 0; k < VEC; ++k) oe[k] = from_f<T>(v[i * VEC + k] * inv * to_f<T>(we[k]));
        __stcs(reinterpret_cast<uint4*>(yr + c), out);
      }
    }
  } else {
    constexpr float LOG2E = 1.4426950408889634f;
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      v[k] *= LOG2E;
      mx = fmaxf(mx, v[k]);
    }
    mx = group_reduce<G, true>(mx, red);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      v[k] = exp2f(v[k] - mx);
      sum += v[k];
    }
    sum = group_reduce<G, false>(sum, red);
    const float inv = 1.f / sum;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * G + g) * VEC;
      if (live && c < N) {
        uint4 out;
        T* oe = reinterpret_cast<T*>(&out);
#pragma unroll
        for (int k = 0; k < VEC; ++k) oe[k] = from_f<T>(v[i * VEC + k] * inv);
        __stcs(reinterpret_cast<uint4*>(yr + c), out);
      }
    }
  }
}

template <int G, int EPT, typename T, int OP>
int launch_cfg(const void* X, const void* W, void* Y, int M, int N, float eps,
               cudaStream_t stream) {
  const long long rows_per_cta = THREADS / G;
  const long long grid = (M + rows_per_cta - 1) / rows_per_cta;
  if (grid > 0x7fffffffLL) return KTA_ERR_UNSUPPORTED;
  return launch_ex(rowop_kernel<G, EPT, T, OP>, dim3(static_cast<unsigned>(grid)), dim3(THREADS),
                   0, stream, 1, static_cast<const T*>(X), static_cast<const T*>(W),
                   static_cast<T*>(Y), M, N, eps);
}

// Threads per row: the smallest power of two >= 32 that keeps a thread at <= 32 elements
// (up to 256 threads, then up to 64 elements).
template <typename T, int OP>
int launch(const void* X, const void* W, void* Y, int64_t M64, int64_t N64, float eps,
           void* stream_v) {
  if (X == nullptr || Y == nullptr || (OP == 0 && W == nullptr)) return KTA_ERR_INVALID_ARG;
  if (M64 <= 0 || N64 <= 0) return KTA_ERR_INVALID_ARG;
  if (OP == 0 && !(eps >= 0.f && std::isfinite(eps))) return KTA_ERR_INVALID_ARG;
  if (M64 > (1LL << 31) - 1 || N64 > THREADS * MAX_EPT) return KTA_ERR_UNSUPPORTED;
  if (N64 % 8 != 0) return KTA_ERR_ALIGN;  // rows are read as 16-byte vectors
  if (!aligned16(X) || !aligned16(Y) || (OP == 0 && !aligned16(W))) return KTA_ERR_ALIGN;
  int s = require_sm100();
  if (s != KTA_OK) return s;
  const int M = static_cast<int>(M64), N = static_cast<int>(N64);
  cudaStream_t st = static_cast<cudaStream_t>(stream_v);
  const int per32 = (N + 31) / 32;  // elements per thread with 32 threads
  if (per32 <= 8) return launch_cfg<32, 8, T, OP>(X, W, Y, M, N, eps, st);
  if (per32 <= 16) return launch_cfg<32, 16, T, OP>(X, W, Y, M, N, eps, st);
  if (per32 <= 32) return launch_cfg<32, 32, T, OP>(X, W, Y, M, N, eps, st);
  if (per32 <= 64) return launch_cfg<64, 32, T, OP>(X, W, Y, M, N, eps, st);
  if (per32 <= 128) return launch_cfg<128, 32, T, OP>(X, W, Y, M, N, eps, st);
  if (per32 <= 256) return launch_cfg<256, 32, T, OP>(X, W, Y, M, N, eps, st);
  return launch_cfg<256, 64, T, OP>(X, W, Y, M, N, eps, st);
}

}  // namespace rowops
}  // namespace kta

extern "C" int kta_rmsnorm_f16(const void* X, const void* W, void* Y, int64_t M, int64_t N,
                               float eps, void* stream) {
  return kta::rowops::launch<__half, 0>(X, W, Y, M, N, eps, stream);
}
extern "C" int kta_rmsnorm_bf16(const void* X, const void* W, void* Y, int64_t M, int64_t N,
                                float eps, void* stream) {
  return kta::rowops::launch<__nv_bfloat16, 0>(X, W, Y, M, N, eps, stream);
}
extern "C" int kta_softmax_f16(const void* X, void* Y, int64_t M, int64_t N, void* stream) {
  return kta::rowops::launch<__half, 1>(X, nullptr, Y, M, N, 0.f, stream);
}
extern "C" int kta_softmax_bf16(const void* X, void* Y, int64_t M, int64_t N, void* stream) {
  return kta::rowops::launch<__nv_bfloat16, 1>(X, nullptr, Y, M, N, 0.f, stream);
}

extern "C" void kta_so_rmsnorm_f16(uint64_t X, uint64_t W, uint64_t Y, int32_t M, int32_t N) {
  kta::set_last_error(kta_rmsnorm_f16(reinterpret_cast<const void*>(X),
                                      reinterpret_cast<const void*>(W), reinterpret_cast<void*>(Y),
                                      M, N, 1e-6f, nullptr));
}
extern "C" void kta_so_softmax_f16(uint64_t X, uint64_t Y, int32_t M, int32_t N) {
  kta::set_last_error(kta_softmax_f16(reinterpret_cast<const void*>(X),
                                      reinterpret_cast<void*>(Y), M, N, nullptr));
}
