// Internal interface between conv2d.cu and gemm_sm100.cu: an implicit-GEMM 2-D convolution on
// the tcgen05 GEMM kernels, whose B tiles are TMA im2col loads of a channels-innermost
// activation instead of tiled loads of a materialised patch matrix.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace ntb {

struct ConvImplicit {
  int dtype;                 // NTB_BF16 or NTB_F16
  const void* w;             // packed weight [K, R * S * CB * 64]: column ((r * S + s) * CB + cb) * 64 + ci
                             // holds w[k, cb * 64 + ci, r, s] (zero for channels >= C)
  int K;                     // output channels
  int CB;                    // 64-channel blocks per filter tap
  const void* x;             // activation [N, H, W, Cs] with channels innermost, Cs >= C
  int64_t x_ws, x_hs, x_ns;  // its strides in elements (w, h, n); multiples of 8
  int Cs, H, W, N;           // channel extent of x's map (C rounded up to 8), input size, images
  int R, S, P, Q;
  int sh, sw, ph, pw, dh, dw;
  void* y;                   // output: image n, channel k, pixel j at y + n * y_ns + k * P * Q + j
  int64_t y_ns;
  const void* bias;          // NULL or [K] with stride bias_s
  int64_t bias_s;
};

// True when the im2col tensor map can describe this convolution (4-D map limits: box corners
// within [-128, 127], traversal steps <= 8) and the operands are 16-byte aligned.
bool conv_implicit_ok(const ConvImplicit& cv);

// Runs y = conv(x, w) + bias for all N images as one batched GEMM (M = K, N = P * Q per image,
// reduction R * S * CB * 64); returns a status.
int conv_implicit_gemm(const ConvImplicit& cv, cudaStream_t st);

}  // namespace ntb
