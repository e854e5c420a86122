// Implicit patch matrix of a KAN convolution (reference kanforge/torch/conv.py:57-85).
//
// A KANConvNd applies one KANLinear per channel group to every receptive
// field: row r of the layer's input is output position (n, o_0, o_1, o_2) and
// column i is (c, k_0, k_1, k_2), the channel inside the group and the kernel
// offset, ordered like the weights of torch.nn.ConvNd.  The value is
//   img[n, c0 + c, o_d * stride_d - pad_d + k_d * dil_d (d = 0..2)]
// or 0 where a position falls in the zero padding.  The fused kernels read
// their x operand through conv_index() instead of a materialised (rows, cols)
// patch matrix; up to three spatial dimensions, unused ones of size 1.
#pragma once

#include "common.cuh"

namespace kf {

struct ConvDev {
  int active;            // 0: x is a plain (rows, I) matrix
  int64_t img_n_stride;  // elements of one image: channels * size_0 * size_1 * size_2
  int c0;                // first image channel of this group
  int size[3], kernel[3], stride[3], pad[3], dil[3], out[3];
};

// Element index of (row, col) in the image, or -1 in the zero padding.
__device__ __forceinline__ int64_t conv_index(const ConvDev& g, int64_t row, int col) {
  const int o2 = (int)(row % g.out[2]);
  int64_t t = row / g.out[2];
  const int o1 = (int)(t % g.out[1]);
  t /= g.out[1];
  const int o0 = (int)(t % g.out[0]);
  const int64_t n = t / g.out[0];
  const int k2 = col % g.kernel[2];
  int u = col / g.kernel[2];
  const int k1 = u % g.kernel[1];
  u /= g.kernel[1];
  const int k0 = u % g.kernel[0];
  const int c = u / g.kernel[0];
  const int p0 = o0 * g.stride[0] - g.pad[0] + k0 * g.dil[0];
  const int p1 = o1 * g.stride[1] - g.pad[1] + k1 * g.dil[1];
  const int p2 = o2 * g.stride[2] - g.pad[2] + k2 * g.dil[2];
  if ((unsigned)p0 >= (unsigned)g.size[0] || (unsigned)p1 >= (unsigned)g.size[1] || (unsigned)p2 >= (unsigned)g.size[2])
    return -1;
  return n * g.img_n_stride + (((int64_t)(g.c0 + c) * g.size[0] + p0) * g.size[1] + p1) * g.size[2] + p2;
}

// bf16 bits of x[row, col]: the plain matrix (row pitch I) or the image.
__device__ __forceinline__ unsigned short x_bits(const __nv_bfloat16* x, const ConvDev& g, int64_t row, int col, int I) {
  const unsigned short* xs = reinterpret_cast<const unsigned short*>(x);
  if (!g.active) return __ldg(xs + row * I + col);
  const int64_t e = conv_index(g, row, col);
  return e >= 0 ? __ldg(xs + e) : (unsigned short)0;
}

__device__ __forceinline__ float x_value(const __nv_bfloat16* x, const ConvDev& g, int64_t row, int col, int I) {
  return __uint_as_float((uint32_t)x_bits(x, g, row, col, I) << 16);
}

}  // namespace kf
