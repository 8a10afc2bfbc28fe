// Load-time weight preparation on the device, and the synthetic generator.
//
// bf16 conversion is round to nearest even, the rounding of the reference's
// f32_to_bf16 (src/tensor/dtype.h:39-46). int8 quantisation restates
// quantize_q8_rows (src/model/cuda/device_weight.cpp:11-26) with the group
// size free: peak = max |w| over the group, scale = peak / 127 (1 when the
// group is all zeros), q = clamp(nearbyint(w / scale), -127, 127). One block
// per row; IEEE division and rintf give the host's bits.
#include "moe_kernels.h"
#include "rms_norm.cuh"

namespace uocr_b200 {
namespace {

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

// bf16 -> fp32 is exact (the bf16 bits are the float's upper half), the
// widening the reference's CheckpointWeights applies to every tensor
// (src/model/weight_source.cpp:21).
__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ src, float* __restrict__ dst, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = __bfloat162float(src[i]);
}

template <typename T>
__device__ __forceinline__ float load_f(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_f<float>(const float* p, int64_t i) {
  return p[i];
}
template <>
__device__ __forceinline__ float load_f<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ w, int64_t cols, int64_t group,
                                                            int8_t* __restrict__ q, float* __restrict__ scales) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const int64_t groups = cols / group;
  const T* src = w + row * cols;
  for (int64_t g = 0; g < groups; ++g) {
    float peak = 0.0f;
    for (int64_t i = threadIdx.x; i < group; i += blockDim.x) peak = fmaxf(peak, fabsf(load_f(src, g * group + i)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = peak;
    __syncthreads();
    if (threadIdx.x == 0) {
      float m = red[0];
      for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
      red[0] = m;
    }
    __syncthreads();
    const float pk = red[0];
    const float scale = pk > 0.0f ? pk / 127.0f : 1.0f;
    if (threadIdx.x == 0) scales[row * groups + g] = scale;
    for (int64_t i = threadIdx.x; i < group; i += blockDim.x) {
      float v = rintf(load_f(src, g * group + i) / scale);
      v = fminf(fmaxf(v, -127.0f), 127.0f);
      q[row * cols + g * group + i] = static_cast<int8_t>(v);
    }
    __syncthreads();
  }
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// value(i) = sigma * ((S + 6) / 65536 - 6), S = the twelve 16-bit words of
// three hashes of (key, i): an Irwin-Hall(12) sum, mean 0 and variance 1
// before the scale. Everything before the final product is exact in fp32.
template <bool kBf16>
__global__ void synth_kernel(uint64_t key, float sigma, int64_t offset, int64_t n, void* out) {
  const uint64_t golden = 0x9E3779B97F4A7C15ull;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < n;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t i = static_cast<uint64_t>(offset + j);
    uint32_t s = 0;
#pragma unroll
    for (uint64_t w = 0; w < 3; ++w) {
      const uint64_t h = mix64(key + (3 * i + w + 1) * golden);
      s += static_cast<uint32_t>(h & 0xffff) + static_cast<uint32_t>((h >> 16) & 0xffff) +
           static_cast<uint32_t>((h >> 32) & 0xffff) + static_cast<uint32_t>(h >> 48);
    }
    const float centred = __fsub_rn(__fmul_rn(static_cast<float>(s + 6u), 1.0f / 65536.0f), 6.0f);
    const float v = __fmul_rn(centred, sigma);
    if (kBf16) {
      static_cast<__nv_bfloat16*>(out)[j] = __float2bfloat16_rn(v);
    } else {
      static_cast<float*>(out)[j] = v;
    }
  }
}

__global__ void add_bias_kernel(float* y, const float* bias, int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[i] = __fadd_rn(y[i], bias[i % cols]);
}

__global__ void fill_f32_kernel(float* dst, float value, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = value;
}

// One block of eight warps per row: its inverse RMS (rms_inv_rows), then the
// normalised row (H % 4 == 0).
__global__ void __launch_bounds__(256) rms_norm_rows_kernel(const float* __restrict__ x, int64_t rows, int H,
                                                            RowNorm norm, float* __restrict__ out) {
  __shared__ double s_part[kNormWarps];
  __shared__ float s_inv[1];
  const int64_t r = blockIdx.x;
  const float* row = x + r * H;
  rms_inv_rows(1, H, norm.eps, [&](int, int q) { return __ldcg(reinterpret_cast<const float4*>(row) + q); }, s_part,
               s_inv);
  const float inv = s_inv[0];
  const float4* src = reinterpret_cast<const float4*>(row);
  const float4* g = reinterpret_cast<const float4*>(norm.gain);
  float4* dst = reinterpret_cast<float4*>(out + r * H);
  for (int q = threadIdx.x; q < H / 4; q += blockDim.x) {
    const float4 v = __ldcg(src + q), w = __ldg(g + q);
    dst[q] = make_float4(rms_apply(v.x, inv, w.x), rms_apply(v.y, inv, w.y), rms_apply(v.z, inv, w.z),
                         rms_apply(v.w, inv, w.w));
  }
}

// out = bf16(float(q) * scale[row]) over [rows, cols] int8 (cols % 16 == 0), 16 weights a thread.
__global__ void dequant_rows_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale, int64_t rows,
                                    int64_t cols, __nv_bfloat16* __restrict__ out) {
  const int64_t n16 = rows * cols / 16;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float s = __ldg(scale + (i * 16) / cols);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(q) + i);
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[8];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float a = static_cast<float>(static_cast<int8_t>(words[w] & 0xffu)) * s;
      const float b = static_cast<float>(static_cast<int8_t>((words[w] >> 8) & 0xffu)) * s;
      const float c = static_cast<float>(static_cast<int8_t>((words[w] >> 16) & 0xffu)) * s;
      const float d = static_cast<float>(static_cast<int8_t>(words[w] >> 24)) * s;
      const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
      o[2 * w] = *reinterpret_cast<const uint32_t*>(&lo);
      o[2 * w + 1] = *reinterpret_cast<const uint32_t*>(&hi);
    }
    uint4* dst = reinterpret_cast<uint4*>(out) + 2 * i;
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

unsigned grid_for(int64_t n) {
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  return static_cast<unsigned>(blocks < 1 ? 1 : blocks);
}

}  // namespace

cudaError_t launch_dequant_rows(const int8_t* q, const float* scale, int64_t rows, int64_t cols, __nv_bfloat16* out,
                                cudaStream_t stream) {
  const int64_t n16 = rows * cols / 16;
  if (n16 <= 0) return cudaSuccess;
  dequant_rows_kernel<<<grid_for(n16), 256, 0, stream>>>(q, scale, rows, cols, out);
  return cudaGetLastError();
}

cudaError_t launch_fill_f32(float* dst, float value, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  fill_f32_kernel<<<grid_for(n), 256, 0, stream>>>(dst, value, n);
  return cudaGetLastError();
}

cudaError_t launch_rms_norm_rows(const float* x, int64_t rows, int H, RowNorm norm, float* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  rms_norm_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(x, rows, H, norm, out);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  f32_to_bf16_kernel<<<grid_for(n), 256, 0, stream>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_bf16_to_f32(const __nv_bfloat16* src, float* dst, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  bf16_to_f32_kernel<<<grid_for(n), 256, 0, stream>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_add_bias(float* y, const float* bias, int64_t rows, int64_t cols, cudaStream_t stream) {
  if (rows * cols == 0) return cudaSuccess;
  add_bias_kernel<<<grid_for(rows * cols), 256, 0, stream>>>(y, bias, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const void* w, bool bf16, int64_t rows, int64_t cols, int64_t group, int8_t* q,
                                 float* scales, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  if (bf16) {
    quantize_rows_kernel<__nv_bfloat16><<<static_cast<unsigned>(rows), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(w), cols, group, q, scales);
  } else {
    quantize_rows_kernel<float><<<static_cast<unsigned>(rows), 256, 0, stream>>>(static_cast<const float*>(w), cols,
                                                                                 group, q, scales);
  }
  return cudaGetLastError();
}

uint64_t synth_key(uint64_t seed, uint64_t stream_id) {
  uint64_t z = seed * 0x9E3779B97F4A7C15ull + stream_id;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

cudaError_t launch_synth(uint64_t seed, uint64_t stream_id, float sigma, int64_t offset, int64_t n, bool bf16,
                         void* out, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const uint64_t key = synth_key(seed, stream_id);
  if (bf16) {
    synth_kernel<true><<<grid_for(n), 256, 0, stream>>>(key, sigma, offset, n, out);
  } else {
    synth_kernel<false><<<grid_for(n), 256, 0, stream>>>(key, sigma, offset, n, out);
  }
  return cudaGetLastError();
}

}  // namespace uocr_b200
