// Bind-time weight packing: layer-blob tensors -> HBM-resident expert layout.
//
// The reference unpacks the blob on the host every layer
// (_common.py:20-58) and its loader upcasts everything to fp32
// (loader/safetensors_storage.py:116-122).  Here the blob is read once on the
// device and each expert matrix is re-encoded:
//   * 16-bit mode: values -> f16 (bf16-valued weights are exact in f16 inside
//     its range; a value beyond +-65504 sets the range flag and bind fails);
//   * int8 mode from a float source: symmetric per-output-row quantisation,
//     scale = fp16(max|w_row| / 127), q = clamp(rint(w / f32(scale)), -127, 127);
//   * int8 mode from an int8 source: copied, fp16 row scales widened to fp32.
// gate_proj / up_proj rows are interleaved in groups of 16, and int8 matrices are
// written tile-major (see DeviceWeights); the caller zeroes int8 matrices first so
// that their padding stays zero.
#include <float.h>

#include "common.cuh"
#include "moe_internal.h"

namespace moe {

MOE_DEV float load_src(const void* p, int dtype, size_t i) {
  switch (dtype) {
    case SRC_F32: return reinterpret_cast<const float*>(p)[i];
    case SRC_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    case SRC_BF16: {
      const uint16_t b = reinterpret_cast<const uint16_t*>(p)[i];
      return __uint_as_float(static_cast<uint32_t>(b) << 16);
    }
    default: return static_cast<float>(reinterpret_cast<const int8_t*>(p)[i]);
  }
}

__device__ float block_max(float v) {
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float r = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
    if (threadIdx.x == 0) red[0] = r;
  }
  __syncthreads();
  const float out = red[0];
  __syncthreads();
  return out;
}

// One CTA per destination row.  f16 rows land at dst + dst_off; int8 rows at
// their tile-major places in the matrix at dst (kpad padded columns).
MOE_DEV void pack_one_row(const void* src, int dtype, size_t src_off, void* dst, size_t dst_off,
                          bool to_int8, float* dst_scale, int dst_row, int cols, size_t kpad,
                          int* range_err) {
  if (to_int8) {
    float amax = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x)
      amax = fmaxf(amax, fabsf(load_src(src, dtype, src_off + c)));
    amax = block_max(amax);
    const __half s16 = __float2half_rn(amax / 127.0f);
    const float s = __half2float(s16);
    if (!isfinite(s) && range_err && threadIdx.x == 0) atomicExch(range_err, 1);
    int8_t* d = reinterpret_cast<int8_t*>(dst);
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      int q = 0;
      if (s > 0.f) {
        const float r = rintf(load_src(src, dtype, src_off + c) / s);
        q = static_cast<int>(fminf(fmaxf(r, -127.f), 127.f));
      }
      d[i8_tile_off(dst_row, c, kpad)] = static_cast<int8_t>(q);
    }
    if (threadIdx.x == 0) dst_scale[dst_row] = s;
  } else {
    __half* d = reinterpret_cast<__half*>(dst) + dst_off;
    bool bad = false;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      const float v = load_src(src, dtype, src_off + c);
      const __half h = __float2half_rn(v);
      bad |= isfinite(v) && !isfinite(__half2float(h));
      d[c] = h;
    }
    if (bad && range_err) atomicExch(range_err, 1);
  }
}

__global__ void __launch_bounds__(256) pack_w13_kernel(const void* gate, const void* up,
                                                       int dtype, void* dst, bool to_int8,
                                                       float* dst_scale, int cols,
                                                       int* range_err) {
  const int pr = blockIdx.x;                 // packed row
  const int g = pr >> 5, w = pr & 31;
  const int src_row = g * 16 + (w & 15);
  const void* src = (w < 16) ? gate : up;
  pack_one_row(src, dtype, static_cast<size_t>(src_row) * cols, dst,
               static_cast<size_t>(pr) * cols, to_int8, dst_scale, pr, cols, i8_pad_cols(cols),
               range_err);
}

__global__ void __launch_bounds__(256) pack_rows_kernel(const void* src, int dtype, void* dst,
                                                        bool to_int8, float* dst_scale,
                                                        int cols, int* range_err) {
  const int r = blockIdx.x;
  pack_one_row(src, dtype, static_cast<size_t>(r) * cols, dst, static_cast<size_t>(r) * cols,
               to_int8, dst_scale, r, cols, i8_pad_cols(cols), range_err);
}

__global__ void __launch_bounds__(256) copy_i8_w13_kernel(const int8_t* gate, const int8_t* up,
                                                          const __half* gs, const __half* us,
                                                          int8_t* dst, float* dst_scale,
                                                          int cols) {
  const int pr = blockIdx.x;
  const int g = pr >> 5, w = pr & 31;
  const int src_row = g * 16 + (w & 15);
  const int8_t* src = ((w < 16) ? gate : up) + static_cast<size_t>(src_row) * cols;
  const size_t kpad = i8_pad_cols(cols);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) dst[i8_tile_off(pr, c, kpad)] = src[c];
  if (threadIdx.x == 0) dst_scale[pr] = __half2float(((w < 16) ? gs : us)[src_row]);
}

__global__ void __launch_bounds__(256) copy_i8_rows_kernel(const int8_t* src, const __half* ss,
                                                           int8_t* dst, float* dst_scale,
                                                           int cols) {
  const int r = blockIdx.x;
  const size_t kpad = i8_pad_cols(cols);
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    dst[i8_tile_off(r, c, kpad)] = src[static_cast<size_t>(r) * cols + c];
  if (threadIdx.x == 0) dst_scale[r] = __half2float(ss[r]);
}

__global__ void to_f32_kernel(const void* src, int dtype, float* dst, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = load_src(src, dtype, static_cast<size_t>(i));
}

cudaError_t launch_pack_rows(const void* src, int src_dtype, void* dst, bool to_int8,
                             float* dst_scale, int rows, int cols, int* range_err,
                             cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  pack_rows_kernel<<<rows, 256, 0, s>>>(src, src_dtype, dst, to_int8, dst_scale, cols, range_err);
  return cudaGetLastError();
}

cudaError_t launch_pack_w13(const void* gate, const void* up, int src_dtype, void* dst,
                            bool to_int8, float* dst_scale, int inter, int cols,
                            int* range_err, cudaStream_t s) {
  if (inter <= 0) return cudaSuccess;
  pack_w13_kernel<<<2 * inter, 256, 0, s>>>(gate, up, src_dtype, dst, to_int8, dst_scale, cols,
                                            range_err);
  return cudaGetLastError();
}

cudaError_t launch_copy_i8_w13(const int8_t* gate, const int8_t* up, const __half* gs,
                               const __half* us, int8_t* dst, float* dst_scale, int inter,
                               int cols, cudaStream_t s) {
  if (inter <= 0) return cudaSuccess;
  copy_i8_w13_kernel<<<2 * inter, 256, 0, s>>>(gate, up, gs, us, dst, dst_scale, cols);
  return cudaGetLastError();
}

cudaError_t launch_copy_i8_rows(const int8_t* src, const __half* ss, int8_t* dst,
                                float* dst_scale, int rows, int cols, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  copy_i8_rows_kernel<<<rows, 256, 0, s>>>(src, ss, dst, dst_scale, cols);
  return cudaGetLastError();
}

cudaError_t launch_to_f32(const void* src, int src_dtype, float* dst, int64_t n,
                          cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int grid = static_cast<int>((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  to_f32_kernel<<<grid, 256, 0, s>>>(src, src_dtype, dst, n);
  return cudaGetLastError();
}

}  // namespace moe
