// rowwise.cu — HBM-bound row kernels around the tied head (sm_100a).
//
// These are the steps either side of the fused tied cross-entropy:
//   * cross-entropy over logits that already exist (the untied
//     CrossEntropyLoss.forward and the sampled-softmax loss), reusing the
//     shard-combine of the tied path for lse and the loss;
//   * RMSNorm forward / backward, the norm that produces the head's input;
//   * the embedding scatter-add that shares the tied matrix's grad, and the
//     AdamW update of that matrix.
// Each kernel reads and writes every element once; the roofline is HBM.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cub/device/device_radix_sort.cuh>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <initializer_list>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "nimbleml_tied_ce.h"

namespace nimble {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Eight consecutive elements as fp32 (16-byte vector loads / stores; the
// pointer must be 16-byte aligned for 16-bit types, 32-byte for fp32).
template <typename T> __device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <> __device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <> __device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) { const float2 f = __half22float2(h[k]); v[2 * k] = f.x; v[2 * k + 1] = f.y; }
}
template <> __device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) { const float2 f = __bfloat1622float2(h[k]); v[2 * k] = f.x; v[2 * k + 1] = f.y; }
}
template <typename T> __device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <> __device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <> __device__ __forceinline__ void store8<__half>(__half* p, const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <> __device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Running (max, sum of exp(x - max)) with one exp per element: the sum is
// rescaled only when the maximum grows.
struct OnlineLse {
  float m = -INFINITY, s = 0.0f;
  __device__ __forceinline__ void add(float v) {
    const float d = v - m;
    if (d > 0.0f) {
      s = s * ex2(-d * kLog2e) + 1.0f;
      m = v;
    } else {
      s += ex2(d * kLog2e);
    }
  }
  // Adds n values with one rescale test for all of them.
  template <int n>
  __device__ __forceinline__ void add_n(const float* v) {
    float vm = v[0];
#pragma unroll
    for (int k = 1; k < n; ++k) vm = fmaxf(vm, v[k]);
    if (vm == -INFINITY) return;  // every value is -inf: nothing to add
    if (vm > m) {
      s = (m == -INFINITY) ? 0.0f : s * ex2((m - vm) * kLog2e);
      m = vm;
    }
    const float ml2 = m * kLog2e;
#pragma unroll
    for (int k = 0; k < n; ++k) s += ex2(fmaf(v[k], kLog2e, -ml2));
  }
  __device__ __forceinline__ void merge(float m2, float s2) {
    if (m2 == -INFINITY) return;
    if (m == -INFINITY) { m = m2; s = s2; return; }
    const float mn = fmaxf(m, m2);
    s = s * ex2((m - mn) * kLog2e) + s2 * ex2((m2 - mn) * kLog2e);
    m = mn;
  }
};

// One block of kRowThreads per row of a [N x V] logits matrix (row pitch ld):
// the row's max, sum-exp and the label's logit (0 when the label is outside
// [0, V)). Each thread folds 16-byte vectors into a running (max, sum-exp);
// warps merge by shuffles, the block through shared memory.
constexpr int kRowThreads = 256;
template <typename T>
__global__ void __launch_bounds__(kRowThreads)
ce_rows_kernel(const T* __restrict__ x, int64_t ld, const int64_t* __restrict__ labels, int64_t N, int64_t V,
               float* __restrict__ out_max, float* __restrict__ out_sum, float* __restrict__ out_tgt) {
  __shared__ float sm_m[kRowThreads / 32], sm_s[kRowThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    const T* r = x + row * ld;
    OnlineLse acc;
    constexpr int kVec = 16 / sizeof(T);
    // Rows of an odd-width matrix start off the 16-byte grid: the first
    // `head` elements go one by one, the rest in 16-byte vectors.
    const int64_t head = min(V, static_cast<int64_t>(((16 - (reinterpret_cast<uintptr_t>(r) & 15)) & 15) / sizeof(T)));
    for (int64_t j = threadIdx.x; j < head; j += kRowThreads) acc.add(to_f<T>(r[j]));
    int64_t j0 = head;
    if (((reinterpret_cast<uintptr_t>(r + head)) & 15) == 0) {
      const int64_t nvec = (V - head) / kVec;
      const uint4* r4 = reinterpret_cast<const uint4*>(r + head);
      auto add_vec = [&](const uint4& u) {
        const T* e = reinterpret_cast<const T*>(&u);
        float v[kVec];
#pragma unroll
        for (int k = 0; k < kVec; ++k) v[k] = to_f<T>(e[k]);
        acc.add_n<kVec>(v);
      };
      // kU 16-byte loads in flight per thread before the first is used.
      constexpr int kU = 4;
      int64_t q = threadIdx.x;
      for (; q + (kU - 1) * kRowThreads < nvec; q += kU * kRowThreads) {
        uint4 u[kU];
#pragma unroll
        for (int i = 0; i < kU; ++i) u[i] = __ldg(r4 + q + i * kRowThreads);
#pragma unroll
        for (int i = 0; i < kU; ++i) add_vec(u[i]);
      }
      for (; q < nvec; q += kRowThreads) add_vec(__ldg(r4 + q));
      j0 = head + nvec * kVec;
    }
    for (int64_t j = j0 + threadIdx.x; j < V; j += kRowThreads) acc.add(to_f<T>(r[j]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, acc.m, off);
      const float s2 = __shfl_xor_sync(0xffffffffu, acc.s, off);
      acc.merge(m2, s2);
    }
    if (lane == 0) {
      sm_m[warp] = acc.m;
      sm_s[warp] = acc.s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      OnlineLse t;
      for (int w = 0; w < kRowThreads / 32; ++w) t.merge(sm_m[w], sm_s[w]);
      out_max[row] = t.m;
      out_sum[row] = t.s;
      const int64_t lab = labels[row];
      out_tgt[row] = (lab >= 0 && lab < V) ? to_f<T>(r[lab]) : 0.0f;
    }
    __syncthreads();
  }
}

// grad[i, j] = (exp(x_ij - lse_i) - [j == y_i]) * grad_scale / n_valid, rows
// with y_i == ignore_index all zero. One warp per row.
template <typename T>
__global__ void __launch_bounds__(kRowThreads)
ce_rows_grad_kernel(const T* __restrict__ x, int64_t ld, const int64_t* __restrict__ labels,
                    const float* __restrict__ lse, int64_t N, int64_t V, int64_t ignore_index,
                    const float* __restrict__ grad_scale, const float* __restrict__ valid_count,
                    T* __restrict__ g, int64_t ldg) {
  const float nv = *valid_count;
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    const int64_t lab = labels[row];
    const bool live = lab != ignore_index && lab >= 0 && lab < V && nv > 0.0f;
    const float scale = live ? *grad_scale / nv : 0.0f;
    const float l2 = live ? lse[row] * kLog2e : 0.0f;
    const T* r = x + row * ld;
    T* o = g + row * ldg;
    constexpr int kVec = 16 / sizeof(T);
    auto grad_one = [&](int64_t j) {
      float p = live ? ex2(fmaf(to_f<T>(r[j]), kLog2e, -l2)) : 0.0f;
      if (j == lab) p -= 1.0f;
      o[j] = from_f<T>(p * scale);
    };
    // Odd-width rows: scalar head up to the 16-byte grid, then vectors, when
    // input and output rows sit at the same offset from it.
    const uintptr_t mis = reinterpret_cast<uintptr_t>(r) & 15;
    const int64_t head = min(V, static_cast<int64_t>(((16 - mis) & 15) / sizeof(T)));
    int64_t j0 = 0;
    if (mis == (reinterpret_cast<uintptr_t>(o) & 15) && (mis % sizeof(T)) == 0) {
      for (int64_t j = threadIdx.x; j < head; j += kRowThreads) grad_one(j);
      const int64_t nvec = (V - head) / kVec;
      const uint4* r4 = reinterpret_cast<const uint4*>(r + head);
      auto grad_vec = [&](const uint4& u, int64_t q) {
        const T* e = reinterpret_cast<const T*>(&u);
        uint4 w;
        T* f = reinterpret_cast<T*>(&w);
#pragma unroll
        for (int k = 0; k < kVec; ++k) {
          float p = live ? ex2(fmaf(to_f<T>(e[k]), kLog2e, -l2)) : 0.0f;
          if (head + q * kVec + k == lab) p -= 1.0f;
          f[k] = from_f<T>(p * scale);
        }
        reinterpret_cast<uint4*>(o + head)[q] = w;
      };
      constexpr int kU = 2;
      int64_t q = threadIdx.x;
      for (; q + (kU - 1) * kRowThreads < nvec; q += kU * kRowThreads) {
        uint4 u[kU];
#pragma unroll
        for (int i = 0; i < kU; ++i) u[i] = __ldg(r4 + q + i * kRowThreads);
#pragma unroll
        for (int i = 0; i < kU; ++i) grad_vec(u[i], q + i * kRowThreads);
      }
      for (; q < nvec; q += kRowThreads) grad_vec(__ldg(r4 + q), q);
      j0 = head + nvec * kVec;
    }
    for (int64_t j = j0 + threadIdx.x; j < V; j += kRowThreads) grad_one(j);
  }
}

// Sampled softmax, one thread per row over its C candidate classes
// (candidate 0 is the true class).
template <typename T>
__global__ void sampled_rows_kernel(const T* __restrict__ x, int64_t ld, const int64_t* __restrict__ cand, int64_t N,
                                    int64_t V, int64_t C, float* __restrict__ out_max, float* __restrict__ out_sum,
                                    float* __restrict__ out_tgt, int* status) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= N) return;
  OnlineLse acc;
  float t = 0.0f;
  bool bad = false;
  for (int64_t c = 0; c < C; ++c) {
    const int64_t k = cand[row * C + c];
    if (k < 0 || k >= V) { bad = true; continue; }
    const float v = to_f<T>(x[row * ld + k]);
    if (c == 0) t = v;
    acc.add(v);
  }
  if (bad && status) atomicOr(status, NIMBLE_STATUS_BAD_LABEL);
  out_max[row] = acc.m;
  out_sum[row] = acc.s;
  out_tgt[row] = t;
}

template <typename T>
__global__ void sampled_rows_grad_kernel(const T* __restrict__ x, int64_t ld, const int64_t* __restrict__ cand,
                                         const int64_t* __restrict__ labels, const float* __restrict__ lse, int64_t N,
                                         int64_t V, int64_t C, int64_t ignore_index,
                                         const float* __restrict__ grad_scale, const float* __restrict__ valid_count,
                                         T* __restrict__ g, int64_t ldg) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= N) return;
  const float nv = *valid_count;
  if (labels[row] == ignore_index || nv <= 0.0f) return;
  const float scale = *grad_scale / nv;
  const float l2 = lse[row] * kLog2e;
  // One thread owns the row, so repeated candidates add up in a fixed order.
  for (int64_t c = 0; c < C; ++c) {
    const int64_t k = cand[row * C + c];
    if (k < 0 || k >= V) continue;
    float p = ex2(fmaf(to_f<T>(x[row * ld + k]), kLog2e, -l2));
    if (c == 0) p -= 1.0f;
    T* dst = g + row * ldg + k;
    *dst = from_f<T>(to_f<T>(*dst) + p * scale);
  }
}

constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) t += red[i];
  return t;
}

template <int THREADS>
__device__ __forceinline__ float block_sum_n(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) t += red[i];
  return t;
}

// y = x / sqrt(mean(x^2) + eps) * gamma, one block per row (grid-stride).
template <typename T, int KMAX>
__global__ void __launch_bounds__(kNormThreads)
rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ gamma, int64_t N, int d, float eps,
                   T* __restrict__ y, float* __restrict__ out_ms, float* __restrict__ out_rms) {
  __shared__ float red[kNormThreads / 32];
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    const T* xr = x + row * d;
    float xv[KMAX];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const int j = threadIdx.x + k * kNormThreads;
      xv[k] = j < d ? to_f<T>(xr[j]) : 0.0f;
      ss = fmaf(xv[k], xv[k], ss);
    }
    const float ms = block_sum(ss, red) / static_cast<float>(d);
    const float rms = sqrtf(ms + eps);
    const float inv = 1.0f / rms;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const int j = threadIdx.x + k * kNormThreads;
      if (j < d) y[row * d + j] = from_f<T>(xv[k] * inv * to_f<T>(gamma[j]));
    }
    if (threadIdx.x == 0) {
      out_ms[row] = ms;
      out_rms[row] = rms;
    }
  }
}

// grad_x = grad*gamma/rms + x * (2/d) * (-1/2) * (sum_j grad_j gamma_j x_j) * (ms+eps)^(-3/2)
// and, per block, partial sums over its rows of grad * x / rms for grad_gamma.
// The incoming grad has its own type GT (fp32 when it comes straight from the
// tied head's fp32 grad_hidden).
template <typename T, typename GT, int KMAX>
__global__ void __launch_bounds__(kNormThreads)
rmsnorm_bwd_kernel(const GT* __restrict__ grad, const T* __restrict__ x, const T* __restrict__ gamma,
                   const float* __restrict__ ms, const float* __restrict__ rms, int64_t N, int d, float eps,
                   T* __restrict__ gx, float* __restrict__ partial) {
  __shared__ float red[kNormThreads / 32];
  float gg[KMAX], gm[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    const int j = threadIdx.x + k * kNormThreads;
    gg[k] = 0.0f;
    gm[k] = j < d ? to_f<T>(gamma[j]) : 0.0f;
  }
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    float gv[KMAX], xv[KMAX];
    float dot = 0.0f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const int j = threadIdx.x + k * kNormThreads;
      gv[k] = j < d ? to_f<GT>(grad[row * d + j]) : 0.0f;
      xv[k] = j < d ? to_f<T>(x[row * d + j]) : 0.0f;
      dot = fmaf(gv[k] * gm[k], xv[k], dot);
    }
    dot = block_sum(dot, red);
    const float inv = 1.0f / rms[row];
    const float msv = ms[row] + eps;
    const float coef = (2.0f / static_cast<float>(d)) * (-0.5f) * dot / (msv * sqrtf(msv));
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const int j = threadIdx.x + k * kNormThreads;
      if (j < d) gx[row * d + j] = from_f<T>(gv[k] * gm[k] * inv + xv[k] * coef);
      gg[k] = fmaf(gv[k], xv[k] * inv, gg[k]);
    }
  }
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    const int j = threadIdx.x + k * kNormThreads;
    if (j < d) partial[static_cast<int64_t>(blockIdx.x) * d + j] = gg[k];
  }
}

// Vector forms of the two RMSNorm kernels for d % 8 == 0 and 16-byte aligned
// rows: thread t of the block owns the 8-element vectors t, t + 256, ...
// (KV of them), so every load and store is 16 bytes wide.
template <typename T, int KV>
__global__ void __launch_bounds__(kNormThreads)
rmsnorm_fwd_vec_kernel(const T* __restrict__ x, const T* __restrict__ gamma, int64_t N, int d, float eps,
                       T* __restrict__ y, float* __restrict__ out_ms, float* __restrict__ out_rms) {
  __shared__ float red[kNormThreads / 32];
  const int nv = d / 8;
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    const T* xr = x + row * d;
    float xv[KV][8];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      const int q = threadIdx.x + k * kNormThreads;
      if (q < nv) {
        load8<T>(xr + 8 * q, xv[k]);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(xv[k][e], xv[k][e], ss);
      }
    }
    const float ms = block_sum(ss, red) / static_cast<float>(d);
    const float rms = sqrtf(ms + eps);
    const float inv = 1.0f / rms;
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      const int q = threadIdx.x + k * kNormThreads;
      if (q < nv) {
        float gv[8], yv[8];
        load8<T>(gamma + 8 * q, gv);
#pragma unroll
        for (int e = 0; e < 8; ++e) yv[e] = xv[k][e] * inv * gv[e];
        store8<T>(y + row * d + 8 * q, yv);
      }
    }
    if (threadIdx.x == 0) {
      out_ms[row] = ms;
      out_rms[row] = rms;
    }
  }
}

template <typename T, typename GT, int KV, int THREADS>
__global__ void __launch_bounds__(THREADS)
rmsnorm_bwd_vec_kernel(const GT* __restrict__ grad, const T* __restrict__ x, const T* __restrict__ gamma,
                       const float* __restrict__ ms, const float* __restrict__ rms, int64_t N, int d, float eps,
                       T* __restrict__ gx, float* __restrict__ partial) {
  __shared__ float red[THREADS / 32];
  const int nv = d / 8;
  float gm[KV][8], gg[KV][8];
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int q = threadIdx.x + k * THREADS;
#pragma unroll
    for (int e = 0; e < 8; ++e) gm[k][e] = gg[k][e] = 0.0f;
    if (q < nv) load8<T>(gamma + 8 * q, gm[k]);
  }
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    float gv[KV][8], xv[KV][8];
    float dot = 0.0f;
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      const int q = threadIdx.x + k * THREADS;
      if (q < nv) {
        load8<GT>(grad + row * d + 8 * q, gv[k]);
        load8<T>(x + row * d + 8 * q, xv[k]);
#pragma unroll
        for (int e = 0; e < 8; ++e) dot = fmaf(gv[k][e] * gm[k][e], xv[k][e], dot);
      }
    }
    dot = block_sum_n<THREADS>(dot, red);
    const float inv = 1.0f / rms[row];
    const float msv = ms[row] + eps;
    const float coef = (2.0f / static_cast<float>(d)) * (-0.5f) * dot / (msv * sqrtf(msv));
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      const int q = threadIdx.x + k * THREADS;
      if (q < nv) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          o[e] = gv[k][e] * gm[k][e] * inv + xv[k][e] * coef;
          gg[k][e] = fmaf(gv[k][e], xv[k][e] * inv, gg[k][e]);
        }
        store8<T>(gx + row * d + 8 * q, o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int q = threadIdx.x + k * THREADS;
    if (q < nv) {
#pragma unroll
      for (int e = 0; e < 8; ++e) partial[static_cast<int64_t>(blockIdx.x) * d + 8 * q + e] = gg[k][e];
    }
  }
}

// grad_gamma[j] (+)= sum over blocks b = 0..G-1 of partial[b, j], in order.
__global__ void sum_partials_kernel(const float* __restrict__ partial, int G, int d, float* __restrict__ out,
                                    int accumulate) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= d) return;
  float s = 0.0f;
  for (int b = 0; b < G; ++b) s += partial[static_cast<int64_t>(b) * d + j];
  out[j] = accumulate ? out[j] + s : s;
}

// Embedding scatter-add, deterministic: each row's id becomes a shard-local
// sort key (ids of other shards and out-of-range ids get the sentinel
// `v_local`), a stable radix sort groups equal keys with their rows in
// ascending order, and one block per group adds those rows to the grad row in
// that order — the loop order of the reference's CPU scatter
// (native/src/scatter.cpp:6-15), so fp32 results do not depend on scheduling.
__global__ void scatter_keys_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t v_off, int64_t v_local,
                                    int64_t vocab, uint32_t* __restrict__ keys, int32_t* __restrict__ rows,
                                    int* status) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t id = ids[i];
    if ((id < 0 || id >= vocab) && status) atomicOr(status, NIMBLE_STATUS_BAD_LABEL);
    const int64_t local = id - v_off;
    keys[i] = (id >= 0 && id < vocab && local >= 0 && local < v_local) ? static_cast<uint32_t>(local)
                                                                       : static_cast<uint32_t>(v_local);
    rows[i] = static_cast<int32_t>(i);
  }
}

template <typename T>
__global__ void scatter_segments_kernel(float* __restrict__ gw, const uint32_t* __restrict__ keys,
                                        const int32_t* __restrict__ rows, const T* __restrict__ go, int64_t n,
                                        uint32_t sentinel, int d, bool vec) {
  for (int64_t b = blockIdx.x; b < n; b += gridDim.x) {
    const uint32_t key = keys[b];
    if (key == sentinel || (b > 0 && keys[b - 1] == key)) continue;  // not the first row of a group
    int64_t e = b + 1;
    while (e < n && keys[e] == key) ++e;
    float* dst = gw + static_cast<int64_t>(key) * d;
    if (vec) {  // 8 columns per thread and step, 16-byte loads and stores
      for (int j = 8 * threadIdx.x; j < d; j += 8 * blockDim.x) {
        float acc[8], g[8];
        load8<float>(dst + j, acc);
        for (int64_t p = b; p < e; ++p) {
          load8<T>(go + static_cast<int64_t>(rows[p]) * d + j, g);
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[k] += g[k];
        }
        store8<float>(dst + j, acc);
      }
      continue;
    }
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
      float acc = dst[j];
      for (int64_t p = b; p < e; ++p) acc += to_f<T>(go[static_cast<int64_t>(rows[p]) * d + j]);
      dst[j] = acc;
    }
  }
}

template <typename G, typename P>
__global__ void adamw_kernel(float* __restrict__ w, const G* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, int64_t n, float lr, float b1, float b2, float bc1, float bc2,
                             float eps, float wd, P* __restrict__ copy) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gi = to_f<G>(g[i]);
    const float mn = b1 * m[i] + (1.0f - b1) * gi;
    const float vn = b2 * v[i] + (1.0f - b2) * gi * gi;
    const float upd = (mn / bc1) / (sqrtf(vn / bc2) + eps);
    const float wn = w[i] * (1.0f - lr * wd) - lr * upd;
    m[i] = mn;
    v[i] = vn;
    w[i] = wn;
    if (copy) copy[i] = from_f<P>(wn);
  }
}

// The same update, 8 elements per thread and step with 16-byte accesses (n a
// multiple of 8, every pointer 16-byte aligned).
template <typename G, typename P>
__global__ void adamw_vec_kernel(float* __restrict__ w, const G* __restrict__ g, float* __restrict__ m,
                                 float* __restrict__ v, int64_t n8, float lr, float b1, float b2, float bc1,
                                 float bc2, float eps, float wd, P* __restrict__ copy) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float wv[8], gv[8], mv[8], vv[8];
    load8<float>(w + 8 * i, wv);
    load8<G>(g + 8 * i, gv);
    load8<float>(m + 8 * i, mv);
    load8<float>(v + 8 * i, vv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float mn = b1 * mv[k] + (1.0f - b1) * gv[k];
      const float vn = b2 * vv[k] + (1.0f - b2) * gv[k] * gv[k];
      const float upd = (mn / bc1) / (sqrtf(vn / bc2) + eps);
      mv[k] = mn;
      vv[k] = vn;
      wv[k] = wv[k] * (1.0f - lr * wd) - lr * upd;
    }
    store8<float>(w + 8 * i, wv);
    store8<float>(m + 8 * i, mv);
    store8<float>(v + 8 * i, vv);
    if (copy) store8<P>(copy + 8 * i, wv);
  }
}

int grid_for(int64_t items, int per_block) {
  const int64_t b = (items + per_block - 1) / per_block;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(b, 148 * 32)));
}

int check_rows(const void* x, int64_t ld, int64_t N, int64_t V, int dtype) {
  if (!valid_dtype(dtype)) return fail(NIMBLE_ERR_INVALID_ARG, "dtype must be NIMBLE_DTYPE_F32, F16 or BF16");
  if (N < 0 || V <= 0 || ld < V) return fail(NIMBLE_ERR_INVALID_ARG, "need n_rows >= 0, n_classes > 0, row pitch >= n_classes");
  if (N > 0 && !x) return fail(NIMBLE_ERR_INVALID_ARG, "null logits pointer");
  return NIMBLE_OK;
}

#define NIMBLE_DISPATCH(dtype, T, ...)                                      \
  switch (dtype) {                                                          \
    case NIMBLE_DTYPE_F32: { using T = float; __VA_ARGS__; break; }         \
    case NIMBLE_DTYPE_F16: { using T = __half; __VA_ARGS__; break; }        \
    default: { using T = __nv_bfloat16; __VA_ARGS__; break; }               \
  }

}  // namespace
}  // namespace nimble

using namespace nimble;

// ------------------------------------------------------- CE over given logits
extern "C" int nimble_ce_logits_forward(const void* logits, int64_t row_pitch, const int64_t* labels, int64_t n_rows,
                                        int64_t n_classes, int dtype, int64_t ignore_index, float* out_max,
                                        float* out_sumexp, float* out_target, float* out_lse, float* out_loss,
                                        float* out_valid_count, int* status, void* stream) {
  if (int rc = check_rows(logits, row_pitch, n_rows, n_classes, dtype)) return rc;
  if (n_rows > 0 && (!labels || !out_max || !out_sumexp || !out_target))
    return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_rows > 0) {
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(n_rows, 148 * 64));
    NIMBLE_DISPATCH(dtype, T,
                    ce_rows_kernel<T><<<grid, kRowThreads, 0, s>>>(
                        static_cast<const T*>(logits), row_pitch, labels, n_rows, n_classes, out_max, out_sumexp,
                        out_target));
    NIMBLE_CUDA_TRY(cudaGetLastError());
  }
  return nimble_tied_ce_combine(out_max, out_sumexp, out_target, 1, labels, n_rows, n_classes, ignore_index,
                                nullptr, nullptr, out_lse, out_loss, out_valid_count, status, stream);
}

extern "C" int nimble_ce_logits_backward(const float* grad_scale, const float* valid_count, const void* logits,
                                         int64_t row_pitch, const int64_t* labels, const float* lse, int64_t n_rows,
                                         int64_t n_classes, int dtype, int64_t ignore_index, void* grad_logits,
                                         int64_t grad_row_pitch, void* stream) {
  if (int rc = check_rows(logits, row_pitch, n_rows, n_classes, dtype)) return rc;
  if (grad_row_pitch < n_classes) return fail(NIMBLE_ERR_INVALID_ARG, "grad row pitch < n_classes");
  if (n_rows == 0) return NIMBLE_OK;
  if (!grad_scale || !valid_count || !labels || !lse || !grad_logits)
    return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(n_rows, 148 * 64));
  NIMBLE_DISPATCH(dtype, T,
                  ce_rows_grad_kernel<T><<<grid, kRowThreads, 0, s>>>(
                      static_cast<const T*>(logits), row_pitch, labels, lse, n_rows, n_classes, ignore_index,
                      grad_scale, valid_count, static_cast<T*>(grad_logits), grad_row_pitch));
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

// ------------------------------------------------------------ sampled softmax
extern "C" int nimble_sampled_ce_forward(const void* logits, int64_t row_pitch, const int64_t* candidates,
                                         const int64_t* labels, int64_t n_rows, int64_t n_classes,
                                         int64_t n_candidates, int dtype, int64_t ignore_index, float* out_max,
                                         float* out_sumexp, float* out_target, float* out_lse, float* out_loss,
                                         float* out_valid_count, int* status, void* stream) {
  if (int rc = check_rows(logits, row_pitch, n_rows, n_classes, dtype)) return rc;
  if (n_candidates <= 0) return fail(NIMBLE_ERR_INVALID_ARG, "n_candidates must be positive");
  if (n_rows > 0 && (!candidates || !labels || !out_max || !out_sumexp || !out_target))
    return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_rows > 0) {
    const unsigned grid = static_cast<unsigned>((n_rows + 127) / 128);
    NIMBLE_DISPATCH(dtype, T,
                    sampled_rows_kernel<T><<<grid, 128, 0, s>>>(static_cast<const T*>(logits), row_pitch, candidates,
                                                                n_rows, n_classes, n_candidates, out_max,
                                                                out_sumexp, out_target, status));
    NIMBLE_CUDA_TRY(cudaGetLastError());
  }
  return nimble_tied_ce_combine(out_max, out_sumexp, out_target, 1, labels, n_rows, n_classes, ignore_index,
                                nullptr, nullptr, out_lse, out_loss, out_valid_count, status, stream);
}

extern "C" int nimble_sampled_ce_backward(const float* grad_scale, const float* valid_count, const void* logits,
                                          int64_t row_pitch, const int64_t* candidates, const int64_t* labels,
                                          const float* lse, int64_t n_rows, int64_t n_classes, int64_t n_candidates,
                                          int dtype, int64_t ignore_index, void* grad_logits, int64_t grad_row_pitch,
                                          void* stream) {
  if (int rc = check_rows(logits, row_pitch, n_rows, n_classes, dtype)) return rc;
  if (grad_row_pitch < n_classes || n_candidates <= 0) return fail(NIMBLE_ERR_INVALID_ARG, "bad sizes");
  if (n_rows == 0) return NIMBLE_OK;
  if (!grad_scale || !valid_count || !candidates || !labels || !lse || !grad_logits)
    return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t es = elem_size(dtype);
  NIMBLE_CUDA_TRY(cudaMemset2DAsync(grad_logits, grad_row_pitch * es, 0, n_classes * es, n_rows, s));
  const unsigned grid = static_cast<unsigned>((n_rows + 127) / 128);
  NIMBLE_DISPATCH(dtype, T,
                  sampled_rows_grad_kernel<T><<<grid, 128, 0, s>>>(
                      static_cast<const T*>(logits), row_pitch, candidates, labels, lse, n_rows, n_classes,
                      n_candidates, ignore_index, grad_scale, valid_count, static_cast<T*>(grad_logits),
                      grad_row_pitch));
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

// -------------------------------------------------------------------- RMSNorm
namespace {
constexpr int kNormMaxD = 32 * kNormThreads;  // 8192
int norm_grid(int64_t N) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(N, 2 * 148))); }
// The vector kernels keep more rows in flight: several blocks per SM.
int norm_vec_grid(int64_t N) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(N, 6 * 148))); }
// 8-element vectors: d a multiple of 8 and every base pointer 16-byte aligned.
bool vec_rows_ok(int d, std::initializer_list<const void*> ptrs) {
  if (d % 8 != 0) return false;
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15) return false;
  return true;
}
}  // namespace

extern "C" int nimble_rmsnorm_forward(const void* x, const void* gamma, int64_t n_rows, int64_t d_model, float eps,
                                      int dtype, void* y, float* out_ms, float* out_rms, void* stream) {
  if (!valid_dtype(dtype)) return fail(NIMBLE_ERR_INVALID_ARG, "bad dtype");
  if (n_rows < 0 || d_model <= 0 || d_model > kNormMaxD)
    return fail(NIMBLE_ERR_INVALID_ARG, "need n_rows >= 0 and 0 < d_model <= 8192");
  if (n_rows == 0) return NIMBLE_OK;
  if (!x || !gamma || !y || !out_ms || !out_rms) return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int d = static_cast<int>(d_model);
  const int grid = norm_grid(n_rows);
  NIMBLE_DISPATCH(dtype, T, {
    const T* xt = static_cast<const T*>(x);
    const T* gt = static_cast<const T*>(gamma);
    T* yt = static_cast<T*>(y);
    if (vec_rows_ok(d, {x, gamma, y})) {
      const int vgrid = norm_vec_grid(n_rows);
      if (d <= 8 * kNormThreads)
        rmsnorm_fwd_vec_kernel<T, 1><<<vgrid, kNormThreads, 0, s>>>(xt, gt, n_rows, d, eps, yt, out_ms, out_rms);
      else if (d <= 16 * kNormThreads)
        rmsnorm_fwd_vec_kernel<T, 2><<<vgrid, kNormThreads, 0, s>>>(xt, gt, n_rows, d, eps, yt, out_ms, out_rms);
      else
        rmsnorm_fwd_vec_kernel<T, 4><<<vgrid, kNormThreads, 0, s>>>(xt, gt, n_rows, d, eps, yt, out_ms, out_rms);
    } else if (d <= 4 * kNormThreads)
      rmsnorm_fwd_kernel<T, 4><<<grid, kNormThreads, 0, s>>>(xt, gt, n_rows, d, eps, yt, out_ms, out_rms);
    else if (d <= 16 * kNormThreads)
      rmsnorm_fwd_kernel<T, 16><<<grid, kNormThreads, 0, s>>>(xt, gt, n_rows, d, eps, yt, out_ms, out_rms);
    else
      rmsnorm_fwd_kernel<T, 32><<<grid, kNormThreads, 0, s>>>(xt, gt, n_rows, d, eps, yt, out_ms, out_rms);
  });
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

extern "C" int nimble_rmsnorm_backward_workspace_size(int64_t n_rows, int64_t d_model, size_t* bytes) {
  if (!bytes || n_rows < 0 || d_model <= 0) return fail(NIMBLE_ERR_INVALID_ARG, "bad arguments");
  *bytes = sizeof(float) * static_cast<size_t>(norm_grid(n_rows)) * static_cast<size_t>(d_model);
  return NIMBLE_OK;
}

extern "C" int nimble_rmsnorm_backward(const void* grad, const void* x, const void* gamma, const float* ms,
                                       const float* rms, int64_t n_rows, int64_t d_model, float eps, int dtype,
                                       int grad_dtype, void* grad_x, float* grad_gamma, int accumulate_grad_gamma,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_dtype(dtype) || !valid_dtype(grad_dtype)) return fail(NIMBLE_ERR_INVALID_ARG, "bad dtype");
  if (n_rows < 0 || d_model <= 0 || d_model > kNormMaxD)
    return fail(NIMBLE_ERR_INVALID_ARG, "need n_rows >= 0 and 0 < d_model <= 8192");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int d = static_cast<int>(d_model);
  if (n_rows == 0) {
    if (grad_gamma && !accumulate_grad_gamma) NIMBLE_CUDA_TRY(cudaMemsetAsync(grad_gamma, 0, sizeof(float) * d, s));
    return NIMBLE_OK;
  }
  if (!grad || !x || !gamma || !ms || !rms || !grad_x || !grad_gamma)
    return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  const bool vec = vec_rows_ok(d, {grad, x, gamma, grad_x});
  const int grid = norm_grid(n_rows);
  if (!workspace || workspace_bytes < sizeof(float) * static_cast<size_t>(grid) * d)
    return fail(NIMBLE_ERR_WORKSPACE, "rmsnorm backward workspace too small");
  float* partial = static_cast<float*>(workspace);
  // The incoming grad is either in the compute dtype or fp32.
  if (grad_dtype != dtype && grad_dtype != NIMBLE_DTYPE_F32)
    return fail(NIMBLE_ERR_INVALID_ARG, "grad_dtype must be the compute dtype or NIMBLE_DTYPE_F32");
  NIMBLE_DISPATCH(dtype, T, {
    const T* xt = static_cast<const T*>(x);
    const T* gm = static_cast<const T*>(gamma);
    T* gxt = static_cast<T*>(grad_x);
    auto launch = [&](auto gt) {
      using GT = std::remove_cv_t<std::remove_pointer_t<decltype(gt)>>;
      if (vec) {  // 512 threads, one or two 8-element vectors each
        constexpr int kT = 2 * kNormThreads;
        if (d <= 8 * kT)
          rmsnorm_bwd_vec_kernel<T, GT, 1, kT><<<grid, kT, 0, s>>>(gt, xt, gm, ms, rms, n_rows, d, eps, gxt, partial);
        else
          rmsnorm_bwd_vec_kernel<T, GT, 2, kT><<<grid, kT, 0, s>>>(gt, xt, gm, ms, rms, n_rows, d, eps, gxt, partial);
        return;
      }
      if (d <= 4 * kNormThreads)
        rmsnorm_bwd_kernel<T, GT, 4><<<grid, kNormThreads, 0, s>>>(gt, xt, gm, ms, rms, n_rows, d, eps, gxt, partial);
      else if (d <= 16 * kNormThreads)
        rmsnorm_bwd_kernel<T, GT, 16><<<grid, kNormThreads, 0, s>>>(gt, xt, gm, ms, rms, n_rows, d, eps, gxt, partial);
      else
        rmsnorm_bwd_kernel<T, GT, 32><<<grid, kNormThreads, 0, s>>>(gt, xt, gm, ms, rms, n_rows, d, eps, gxt, partial);
    };
    if (grad_dtype == NIMBLE_DTYPE_F32)
      launch(static_cast<const float*>(grad));
    else
      launch(static_cast<const T*>(grad));
  });
  NIMBLE_CUDA_TRY(cudaGetLastError());
  sum_partials_kernel<<<(d + 255) / 256, 256, 0, s>>>(partial, grid, d, grad_gamma, accumulate_grad_gamma);
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

// ------------------------------------------------ embedding grad and AdamW
namespace {
// Workspace of the scatter-add: keys and row indices in and out of the
// stable radix sort, then the sort's own temporary storage.
struct ScatterLayout {
  size_t keys_in = 0, keys_out = 0, rows_in = 0, rows_out = 0, temp = 0, temp_bytes = 0, total = 0;
};
int key_bits(int64_t v_local) {
  int bits = 1;
  while ((int64_t(1) << bits) <= v_local) ++bits;  // keys 0..v_local inclusive
  return bits;
}
int scatter_layout(int64_t n, int64_t v_local, ScatterLayout* L) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  size_t off = 0;
  L->keys_in = off; off = up(off + sizeof(uint32_t) * n);
  L->keys_out = off; off = up(off + sizeof(uint32_t) * n);
  L->rows_in = off; off = up(off + sizeof(int32_t) * n);
  L->rows_out = off; off = up(off + sizeof(int32_t) * n);
  size_t temp = 0;
  NIMBLE_CUDA_TRY(cub::DeviceRadixSort::SortPairs(nullptr, temp, static_cast<const uint32_t*>(nullptr),
                                                  static_cast<uint32_t*>(nullptr), static_cast<const int32_t*>(nullptr),
                                                  static_cast<int32_t*>(nullptr), static_cast<int>(n), 0,
                                                  key_bits(v_local)));
  L->temp = off;
  L->temp_bytes = temp;
  off = up(off + temp);
  L->total = off;
  return NIMBLE_OK;
}
}  // namespace

extern "C" int nimble_embedding_scatter_add_workspace_size(int64_t n_rows, int64_t vocab_rows, size_t* bytes) {
  if (!bytes || n_rows < 0 || n_rows > INT32_MAX || vocab_rows <= 0 || vocab_rows >= INT32_MAX)
    return fail(NIMBLE_ERR_INVALID_ARG, "need 0 <= n_rows < 2^31, 0 < vocab_rows < 2^31 and a bytes pointer");
  ScatterLayout L;
  if (n_rows == 0) {
    *bytes = 0;
    return NIMBLE_OK;
  }
  if (int rc = scatter_layout(n_rows, vocab_rows, &L)) return rc;
  *bytes = L.total;
  return NIMBLE_OK;
}

extern "C" int nimble_embedding_scatter_add(float* grad_weights, const int64_t* ids, const void* grad_out,
                                            int64_t n_rows, int64_t vocab_offset, int64_t vocab_rows,
                                            int64_t vocab_size, int64_t d_model, int grad_out_dtype,
                                            void* workspace, size_t workspace_bytes, int* status, void* stream) {
  if (!valid_dtype(grad_out_dtype)) return fail(NIMBLE_ERR_INVALID_ARG, "bad dtype");
  if (n_rows < 0 || n_rows > INT32_MAX || vocab_rows <= 0 || vocab_rows >= INT32_MAX || vocab_size <= 0 ||
      vocab_offset < 0 || vocab_offset + vocab_rows > vocab_size || d_model <= 0 || d_model > INT32_MAX)
    return fail(NIMBLE_ERR_INVALID_ARG, "bad sizes");
  if (n_rows == 0) return NIMBLE_OK;
  if (!grad_weights || !ids || !grad_out) return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  ScatterLayout L;
  if (int rc = scatter_layout(n_rows, vocab_rows, &L)) return rc;
  if (!workspace || workspace_bytes < L.total) return fail(NIMBLE_ERR_WORKSPACE, "scatter-add workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* keys_in = reinterpret_cast<uint32_t*>(ws + L.keys_in);
  uint32_t* keys_out = reinterpret_cast<uint32_t*>(ws + L.keys_out);
  int32_t* rows_in = reinterpret_cast<int32_t*>(ws + L.rows_in);
  int32_t* rows_out = reinterpret_cast<int32_t*>(ws + L.rows_out);
  scatter_keys_kernel<<<grid_for(n_rows, 256), 256, 0, s>>>(ids, n_rows, vocab_offset, vocab_rows, vocab_size, keys_in,
                                                            rows_in, status);
  NIMBLE_CUDA_TRY(cudaGetLastError());
  size_t temp = L.temp_bytes;
  NIMBLE_CUDA_TRY(cub::DeviceRadixSort::SortPairs(ws + L.temp, temp, keys_in, keys_out, rows_in, rows_out,
                                                  static_cast<int>(n_rows), 0, key_bits(vocab_rows), s));
  const int grid = static_cast<int>(std::min<int64_t>(n_rows, 148 * 16));
  const int threads = d_model >= 256 ? 256 : 128;
  NIMBLE_DISPATCH(grad_out_dtype, T,
                  scatter_segments_kernel<T><<<grid, threads, 0, s>>>(
                      grad_weights, keys_out, rows_out, static_cast<const T*>(grad_out), n_rows,
                      static_cast<uint32_t>(vocab_rows), static_cast<int>(d_model),
                      vec_rows_ok(static_cast<int>(d_model), {grad_weights, grad_out})));
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

extern "C" int nimble_adamw_step(float* weights, const void* grad, int grad_dtype, float* exp_avg, float* exp_avg_sq,
                                 int64_t n, float lr, float beta1, float beta2, float bias_correction1,
                                 float bias_correction2, float eps, float weight_decay, void* weights_copy,
                                 int weights_copy_dtype, void* stream) {
  if (!valid_dtype(grad_dtype) || (weights_copy && !valid_dtype(weights_copy_dtype)))
    return fail(NIMBLE_ERR_INVALID_ARG, "bad dtype");
  if (n < 0) return fail(NIMBLE_ERR_INVALID_ARG, "bad size");
  if (n == 0) return NIMBLE_OK;
  if (!weights || !grad || !exp_avg || !exp_avg_sq) return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(n, 256);
  const int cdt = weights_copy ? weights_copy_dtype : NIMBLE_DTYPE_F32;
  const bool vec = n % 8 == 0 && vec_rows_ok(8, {weights, grad, exp_avg, exp_avg_sq, weights_copy});
  NIMBLE_DISPATCH(grad_dtype, G, {
    NIMBLE_DISPATCH(cdt, P, {
      if (vec)
        adamw_vec_kernel<G, P><<<grid_for(n / 8, 256), 256, 0, s>>>(
            weights, static_cast<const G*>(grad), exp_avg, exp_avg_sq, n / 8, lr, beta1, beta2, bias_correction1,
            bias_correction2, eps, weight_decay, static_cast<P*>(weights_copy));
      else
        adamw_kernel<G, P><<<grid, 256, 0, s>>>(weights, static_cast<const G*>(grad), exp_avg, exp_avg_sq, n, lr,
                                                beta1, beta2, bias_correction1, bias_correction2, eps, weight_decay,
                                                static_cast<P*>(weights_copy));
    });
  });
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}
