// Element-wise kernels of the Qwen2 decoder body that surround the attention
// path: RMSNorm, residual add + RMSNorm, SiLU(gate) * up, and the greedy
// argmax over the vocabulary.
//
// In the reference engine these are Hugging Face Qwen2 modules
// (Qwen2RMSNorm, the decoder layer's residual adds, Qwen2MLP's act_fn(gate) *
// up) that torch.compile fuses into a few generated kernels; eagerly they
// are about 20 launches per layer. Here each is one launch. They follow
// torch's fp16 recipe operation for operation so the results match HF's
// modules: fp16 + fp16 residual adds rounded once; RMSNorm in fp32
// (sum of squares, times 1/hidden, + eps, rsqrt, scale), rounded to fp16,
// then multiplied by the fp16 weight and rounded again; SiLU in fp32 as
// x / (1 + exp(-x)), rounded to fp16, times up, rounded again. Only the order
// of the sum of squares differs from torch's reduction.
//
// This file is compiled WITHOUT --use_fast_math (expf, the division and
// rsqrtf keep their IEEE / library accuracy), separately from the attention
// kernels.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include "cie_host.h"
#include "cie_model_ops.h"

namespace cie {
namespace body {

constexpr int kWarpsPerCta = 4;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row; 8 halves (16 bytes) per lane per chunk. With `delta`,
// h = h + delta is written back to h first (the residual stream).
// kChunks > 0: the row is held in registers (chunk c of lane l is
// l + 32 i, i < kChunks, so hidden <= 256 kChunks) and every load of h, delta
// and the weight is issued before the first use: one memory round trip per
// row. kChunks == 0: any width, the row is read twice.
template <bool kAdd, int kChunks>
__global__ void __launch_bounds__(32 * kWarpsPerCta)
    rms_norm_kernel(__half* __restrict__ h, const __half* __restrict__ delta,
                    const __half* __restrict__ w, __half* __restrict__ out, int64_t rows,
                    int hidden, int64_t h_stride, int64_t d_stride, int64_t o_stride,
                    float eps) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  __half* hr = h + row * h_stride;
  const __half* dr = kAdd ? delta + row * d_stride : nullptr;
  __half* orow = out + row * o_stride;
  const int chunks = hidden >> 3;
  const float inv_n = 1.0f / static_cast<float>(hidden);
  if constexpr (kChunks > 0) {
    uint4 x[kChunks], d[kChunks], wv[kChunks];
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = lane + 32 * i;
      if (c < chunks) {
        x[i] = reinterpret_cast<const uint4*>(hr)[c];
        if (kAdd) d[i] = reinterpret_cast<const uint4*>(dr)[c];
        wv[i] = reinterpret_cast<const uint4*>(w)[c];
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = lane + 32 * i;
      if (c < chunks) {
        __half2* xh = reinterpret_cast<__half2*>(&x[i]);
        if (kAdd) {
          const __half2* dh = reinterpret_cast<const __half2*>(&d[i]);
#pragma unroll
          for (int k = 0; k < 4; ++k) xh[k] = __hadd2_rn(xh[k], dh[k]);
          reinterpret_cast<uint4*>(hr)[c] = x[i];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(xh[k]);
          ss = fmaf(f.x, f.x, ss);
          ss = fmaf(f.y, f.y, ss);
        }
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss * inv_n + eps);
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = lane + 32 * i;
      if (c < chunks) {
        const __half2* xh = reinterpret_cast<const __half2*>(&x[i]);
        const __half2* wh = reinterpret_cast<const __half2*>(&wv[i]);
        uint4 y;
        __half2* yh = reinterpret_cast<__half2*>(&y);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(xh[k]);
          yh[k] = __hmul2_rn(wh[k], __floats2half2_rn(f.x * r, f.y * r));
        }
        reinterpret_cast<uint4*>(orow)[c] = y;
      }
    }
  } else {
    float ss = 0.f;
    for (int c = lane; c < chunks; c += 32) {
      uint4 x = reinterpret_cast<const uint4*>(hr)[c];
      __half2* xh = reinterpret_cast<__half2*>(&x);
      if (kAdd) {
        const uint4 d = reinterpret_cast<const uint4*>(dr)[c];
        const __half2* dh = reinterpret_cast<const __half2*>(&d);
#pragma unroll
        for (int k = 0; k < 4; ++k) xh[k] = __hadd2_rn(xh[k], dh[k]);
        reinterpret_cast<uint4*>(hr)[c] = x;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(xh[k]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss * inv_n + eps);
    for (int c = lane; c < chunks; c += 32) {
      // this lane wrote chunk c of h above: its own store is visible to it
      const uint4 x = reinterpret_cast<const uint4*>(hr)[c];
      const uint4 wv = reinterpret_cast<const uint4*>(w)[c];
      const __half2* xh = reinterpret_cast<const __half2*>(&x);
      const __half2* wh = reinterpret_cast<const __half2*>(&wv);
      uint4 y;
      __half2* yh = reinterpret_cast<__half2*>(&y);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(xh[k]);
        yh[k] = __hmul2_rn(wh[k], __floats2half2_rn(f.x * r, f.y * r));
      }
      reinterpret_cast<uint4*>(orow)[c] = y;
    }
  }
}

// out[r, i] = half(silu(gate[r, i])) * up[r, i], 8 elements per thread.
__global__ void silu_mul_kernel(const __half* __restrict__ gate, const __half* __restrict__ up,
                                __half* __restrict__ out, int64_t rows, int inter,
                                int64_t g_stride, int64_t u_stride, int64_t o_stride) {
  const int chunks = inter >> 3;
  const int64_t total = rows * chunks;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / chunks;
    const int c = static_cast<int>(e - r * chunks);
    const uint4 g = reinterpret_cast<const uint4*>(gate + r * g_stride)[c];
    const uint4 u = reinterpret_cast<const uint4*>(up + r * u_stride)[c];
    const __half2* gh = reinterpret_cast<const __half2*>(&g);
    const __half2* uh = reinterpret_cast<const __half2*>(&u);
    uint4 y;
    __half2* yh = reinterpret_cast<__half2*>(&y);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __half22float2(gh[i]);
      const __half2 s = __floats2half2_rn(x.x / (1.0f + expf(-x.x)), x.y / (1.0f + expf(-x.y)));
      yh[i] = __hmul2_rn(s, uh[i]);
    }
    reinterpret_cast<uint4*>(out + r * o_stride)[c] = y;
  }
}

// Index of the largest value of each row (the first one when several are
// equal; a NaN counts as larger than any number, the first NaN wins), as
// torch.argmax. Two launches: kArgmaxParts CTAs per row each reduce one
// contiguous part of the row to a (value, index) partial, then one warp per
// row reduces the partials.
constexpr int kArgmaxThreads = 256;
constexpr int kArgmaxParts = 16;

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  // v at index i beats bv at index bi: NaN above everything, then larger, then earlier
  const bool vn = v != v, bn = bv != bv;
  if (vn != bn) return vn;
  if (!vn && v != bv) return v > bv;
  return i < bi;
}

__device__ __forceinline__ void warp_best(float& bv, int& bi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
}

// kVec: rows 16-byte aligned (8 values per load); otherwise one value per load.
template <bool kVec>
__global__ void __launch_bounds__(kArgmaxThreads)
    argmax_part_kernel(const __half* __restrict__ x, float2* __restrict__ part, int n,
                       int64_t stride) {
  const __half* row = x + static_cast<int64_t>(blockIdx.x) * stride;
  // part p covers chunks [p * per, (p + 1) * per) of 8 values (the tail of
  // the row, and unaligned rows, value by value)
  const int chunks = n >> 3;
  const int per = (chunks + kArgmaxParts - 1) / kArgmaxParts;
  const int c_lo = blockIdx.y * per, c_hi = min(chunks, c_lo + per);
  // start from the part's first value so that a part of -inf keeps its first index
  float bv = -CUDART_INF_F;
  int bi = 0x7fffffff;
  if (kVec && c_lo < c_hi && threadIdx.x == 0) {
    bv = __half2float(row[c_lo * 8]);
    bi = c_lo * 8;
  }
  if (kVec) {
    constexpr int kUnroll = 4;
    for (int c0 = c_lo + threadIdx.x; c0 < c_hi; c0 += kUnroll * kArgmaxThreads) {
      uint4 u[kUnroll];
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const int c = c0 + j * kArgmaxThreads;
        u[j] = c < c_hi ? __ldg(reinterpret_cast<const uint4*>(row) + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const int c = c0 + j * kArgmaxThreads;
        if (c >= c_hi) break;
        const __half2* h = reinterpret_cast<const __half2*>(&u[j]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // this thread visits its indices in increasing order: a strictly
          // larger value (or a first NaN) is the only way to replace the best
          const float2 f = __half22float2(h[e]);
          if (f.x > bv || (f.x != f.x && bv == bv)) { bv = f.x; bi = c * 8 + 2 * e; }
          if (f.y > bv || (f.y != f.y && bv == bv)) { bv = f.y; bi = c * 8 + 2 * e + 1; }
        }
      }
    }
  }
  // values not covered by 16-byte loads: the row tail (last part), or all of
  // this part's range when rows are unaligned
  const int v_lo = kVec ? (blockIdx.y == kArgmaxParts - 1 ? chunks * 8 : n) : c_lo * 8;
  const int v_hi = kVec ? n : (blockIdx.y == kArgmaxParts - 1 ? n : c_hi * 8);
  for (int i = v_lo + threadIdx.x; i < v_hi; i += kArgmaxThreads) {
    const float f = __half2float(row[i]);
    if (better(f, i, bv, bi)) { bv = f; bi = i; }
  }
  warp_best(bv, bi);
  __shared__ float s_v[kArgmaxThreads / 32];
  __shared__ int s_i[kArgmaxThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_v[warp] = bv;
    s_i[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    bv = lane < kArgmaxThreads / 32 ? s_v[lane] : -CUDART_INF_F;
    bi = lane < kArgmaxThreads / 32 ? s_i[lane] : 0x7fffffff;
    warp_best(bv, bi);
    if (lane == 0)
      part[static_cast<int64_t>(blockIdx.x) * kArgmaxParts + blockIdx.y] =
          make_float2(bv, __int_as_float(bi));
  }
}

__global__ void argmax_final_kernel(const float2* __restrict__ part, int64_t* __restrict__ out) {
  const int lane = threadIdx.x;
  float bv = -CUDART_INF_F;
  int bi = 0x7fffffff;
  if (lane < kArgmaxParts) {
    const float2 p = part[static_cast<int64_t>(blockIdx.x) * kArgmaxParts + lane];
    bv = p.x;
    bi = __float_as_int(p.y);
  }
  warp_best(bv, bi);
  if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
}

inline bool aligned_rows(const void* p, int64_t stride) {
  return aligned16(p) && (stride % 8) == 0;
}

}  // namespace body
}  // namespace cie

extern "C" {

int cie_rms_norm(void* h, const void* delta, const void* weight, void* out, int64_t rows,
                 int hidden, int64_t h_stride, int64_t delta_stride, int64_t out_stride,
                 float eps, cie_stream_t stream) {
  using namespace cie;
  using namespace cie::body;
  if (rows < 0 || hidden < 0) return fail(CIE_ERR_INVALID_ARGUMENT, "negative rows / hidden");
  if (rows == 0 || hidden == 0) return CIE_OK;
  if (!h || !weight || !out) return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (hidden % 8) return fail(CIE_ERR_UNSUPPORTED, "hidden %d must be a multiple of 8", hidden);
  if (!aligned_rows(h, h_stride) || !aligned_rows(out, out_stride) || !aligned16(weight) ||
      (delta && !aligned_rows(delta, delta_stride)))
    return fail(CIE_ERR_ALIGNMENT, "rows must start on 16-byte boundaries");
  if (h_stride < hidden || out_stride < hidden || (delta && delta_stride < hidden))
    return fail(CIE_ERR_INVALID_ARGUMENT, "row strides must be >= hidden");
  if (!(eps >= 0.f)) return fail(CIE_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  const int64_t ctas = (rows + kWarpsPerCta - 1) / kWarpsPerCta;
  if (ctas > 0x7fffffff) return fail(CIE_ERR_OVERFLOW, "too many rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* hp = static_cast<__half*>(h);
  auto* op = static_cast<__half*>(out);
  const auto* wp = static_cast<const __half*>(weight);
  const auto* dp = static_cast<const __half*>(delta);
  const unsigned grid = static_cast<unsigned>(ctas);
  const int chunks_per_lane = (hidden / 8 + 31) / 32;
  auto launch = [&](auto kernel) {
    kernel<<<grid, 32 * kWarpsPerCta, 0, s>>>(hp, dp, wp, op, rows, hidden, h_stride,
                                              delta ? delta_stride : 0, out_stride, eps);
  };
  if (delta) {
    if (chunks_per_lane <= 4) launch(rms_norm_kernel<true, 4>);
    else if (chunks_per_lane <= 8) launch(rms_norm_kernel<true, 8>);
    else launch(rms_norm_kernel<true, 0>);
  } else {
    if (chunks_per_lane <= 4) launch(rms_norm_kernel<false, 4>);
    else if (chunks_per_lane <= 8) launch(rms_norm_kernel<false, 8>);
    else launch(rms_norm_kernel<false, 0>);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "rms_norm launch: %s", cudaGetErrorString(e));
  return CIE_OK;
}

int cie_silu_mul(const void* gate, const void* up, void* out, int64_t rows, int inter,
                 int64_t gate_stride, int64_t up_stride, int64_t out_stride,
                 cie_stream_t stream) {
  using namespace cie;
  using namespace cie::body;
  if (rows < 0 || inter < 0) return fail(CIE_ERR_INVALID_ARGUMENT, "negative rows / size");
  if (rows == 0 || inter == 0) return CIE_OK;
  if (!gate || !up || !out) return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (inter % 8) return fail(CIE_ERR_UNSUPPORTED, "size %d must be a multiple of 8", inter);
  if (!aligned_rows(gate, gate_stride) || !aligned_rows(up, up_stride) ||
      !aligned_rows(out, out_stride))
    return fail(CIE_ERR_ALIGNMENT, "rows must start on 16-byte boundaries");
  if (gate_stride < inter || up_stride < inter || out_stride < inter)
    return fail(CIE_ERR_INVALID_ARGUMENT, "row strides must be >= size");
  const int64_t total = rows * (inter / 8);
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  const unsigned blocks = static_cast<unsigned>(want < 8L * sm_count() ? want : 8L * sm_count());
  silu_mul_kernel<<<blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(gate), static_cast<const __half*>(up), static_cast<__half*>(out),
      rows, inter, gate_stride, up_stride, out_stride);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "silu_mul launch: %s", cudaGetErrorString(e));
  return CIE_OK;
}

size_t cie_argmax_workspace_bytes(int64_t rows) {
  return rows <= 0 ? 0 : static_cast<size_t>(rows) * cie::body::kArgmaxParts * 2 * sizeof(float);
}

int cie_argmax_rows(const void* x, int64_t rows, int n, int64_t stride, int64_t* out,
                    void* workspace, size_t workspace_bytes, cie_stream_t stream) {
  using namespace cie;
  using namespace cie::body;
  if (rows < 0 || n < 0) return fail(CIE_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0) return CIE_OK;
  if (!x || !out || n == 0) return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer or empty row");
  if (rows > 65535) return fail(CIE_ERR_UNSUPPORTED, "rows %lld > 65535", (long long)rows);
  if (stride < n) return fail(CIE_ERR_INVALID_ARGUMENT, "row stride < n");
  if ((reinterpret_cast<uintptr_t>(x) & 1) != 0)
    return fail(CIE_ERR_ALIGNMENT, "x must be 2-byte aligned");
  if (workspace == nullptr || workspace_bytes < cie_argmax_workspace_bytes(rows))
    return fail(CIE_ERR_WORKSPACE, "argmax needs %zu workspace bytes",
                cie_argmax_workspace_bytes(rows));
  if ((reinterpret_cast<uintptr_t>(workspace) & 7) != 0)
    return fail(CIE_ERR_ALIGNMENT, "workspace must be 8-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float2* part = static_cast<float2*>(workspace);
  const dim3 grid(static_cast<unsigned>(rows), kArgmaxParts);
  if (aligned_rows(x, stride))
    argmax_part_kernel<true><<<grid, kArgmaxThreads, 0, s>>>(static_cast<const __half*>(x), part,
                                                             n, stride);
  else
    argmax_part_kernel<false><<<grid, kArgmaxThreads, 0, s>>>(static_cast<const __half*>(x), part,
                                                              n, stride);
  argmax_final_kernel<<<static_cast<unsigned>(rows), 32, 0, s>>>(part, out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "argmax launch: %s", cudaGetErrorString(e));
  return CIE_OK;
}

}  // extern "C"
