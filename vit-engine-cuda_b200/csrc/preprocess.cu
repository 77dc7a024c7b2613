// Image preprocessing on the GPU: the step before the ViT forward in the
// reference (vit_cuda/model.py:180-188, scripts/eval_imagenette.py:210-215:
// torchvision Resize(256) -> CenterCrop(224) -> ToTensor -> Normalize).
//
// Input: a batch of equal-size 8-bit RGB images, HWC, as decoders produce
// them. Output: fp32 [B][3][crop][crop], (x / 255 - mean[c]) / std[c].
//
// Resize is antialiased bilinear resampling, the separable triangle filter
// torchvision applies (antialias=True; PIL's BILINEAR resize is the same
// filter): along an axis with scale s = in / out, output index i has centre
// c = s * (i + 0.5); the filter spans max(s, 1) input pixels on each side of
// c, tap j (input index) weighs max(0, 1 - |(j - c + 0.5) / max(s, 1)|), and
// the weights are normalised to sum to one. Only the cropped window of the
// resized image is computed: one thread per output pixel, all three channels,
// the two 1-D weight sets evaluated on the fly (no workspace). Arithmetic is
// fp32 throughout (torchvision's tensor path); PIL's uint8 path additionally
// rounds to 8 bits between its two passes.
#include <math.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "engine.h"
#include "vitb200.h"

namespace vitb200 {

struct PreArgs {
  int B, H, W;
  int64_t img_stride;  // bytes between images
  int crop;
  int top, left;       // crop offset inside the resized image
  float sy, sx;        // input / resized size per axis
  float mean[3], inv_std[3];
};

// Input window and normalisation of the 1-D filter for output index i.
__device__ __forceinline__ void aa_window(float s, int i, int in_size, int& lo, int& n,
                                          float& centre, float& inv_support_scale, float& inv_total) {
  const float support = s >= 1.f ? s : 1.f;
  inv_support_scale = 1.f / support;
  centre = s * (static_cast<float>(i) + 0.5f);
  lo = max(static_cast<int>(centre - support + 0.5f), 0);
  const int hi = min(static_cast<int>(centre + support + 0.5f), in_size);
  n = hi - lo;
  float total = 0.f;
  for (int j = 0; j < n; ++j)
    total += fmaxf(0.f, 1.f - fabsf((static_cast<float>(j + lo) - centre + 0.5f) * inv_support_scale));
  inv_total = total > 0.f ? 1.f / total : 0.f;
}

__global__ void preprocess_kernel(const uint8_t* __restrict__ img, float* __restrict__ out,
                                  PreArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t per_img = static_cast<int64_t>(a.crop) * a.crop;
  const int64_t total = per_img * a.B;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(idx / per_img);
    const int rem = static_cast<int>(idx - static_cast<int64_t>(b) * per_img);
    const int y = rem / a.crop, x = rem - (rem / a.crop) * a.crop;
    int y0, ny, x0, nx;
    float cy, cx, iy, ix, ty, tx;
    aa_window(a.sy, y + a.top, a.H, y0, ny, cy, iy, ty);
    aa_window(a.sx, x + a.left, a.W, x0, nx, cx, ix, tx);
    const uint8_t* base = img + static_cast<int64_t>(b) * a.img_stride;
    float acc[3] = {0.f, 0.f, 0.f};
    for (int r = 0; r < ny; ++r) {
      const float wy =
          fmaxf(0.f, 1.f - fabsf((static_cast<float>(r + y0) - cy + 0.5f) * iy)) * ty;
      const uint8_t* row = base + (static_cast<int64_t>(y0 + r) * a.W + x0) * 3;
      float racc[3] = {0.f, 0.f, 0.f};
      for (int q = 0; q < nx; ++q) {
        const float wx =
            fmaxf(0.f, 1.f - fabsf((static_cast<float>(q + x0) - cx + 0.5f) * ix)) * tx;
        racc[0] = fmaf(wx, static_cast<float>(row[3 * q]), racc[0]);
        racc[1] = fmaf(wx, static_cast<float>(row[3 * q + 1]), racc[1]);
        racc[2] = fmaf(wx, static_cast<float>(row[3 * q + 2]), racc[2]);
      }
      acc[0] = fmaf(wy, racc[0], acc[0]);
      acc[1] = fmaf(wy, racc[1], acc[1]);
      acc[2] = fmaf(wy, racc[2], acc[2]);
    }
    float* o = out + static_cast<int64_t>(b) * 3 * per_img + rem;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      o[c * per_img] = (acc[c] * (1.f / 255.f) - a.mean[c]) * a.inv_std[c];
  }
}

}  // namespace vitb200

using namespace vitb200;

extern "C" int vitb200_preprocess(const uint8_t* images, int B, int H, int W, int64_t image_stride,
                                  int resize_short, int crop, const float* mean, const float* stdv,
                                  float* out, void* stream) {
  if (B < 0 || H <= 0 || W <= 0 || resize_short <= 0 || crop <= 0 || !mean || !stdv)
    return VITB200_E_INVALID_ARG;
  if (image_stride < static_cast<int64_t>(H) * W * 3) return VITB200_E_INVALID_ARG;
  if (B == 0) return 0;
  if (!images || !out) return VITB200_E_INVALID_ARG;
  // Resized size: the shorter side becomes resize_short, the longer one
  // floor(resize_short * long / short), as torchvision's Resize(int).
  const bool w_short = W <= H;
  const int shrt = w_short ? W : H, lng = w_short ? H : W;
  const int new_long = static_cast<int>(static_cast<double>(resize_short) * lng / shrt);
  const int RH = w_short ? new_long : resize_short;
  const int RW = w_short ? resize_short : new_long;
  if (RH < crop || RW < crop) return VITB200_E_UNSUPPORTED;  // torchvision would pad
  PreArgs a;
  a.B = B;
  a.H = H;
  a.W = W;
  a.img_stride = image_stride;
  a.crop = crop;
  // CenterCrop offsets round half to even (Python's round()).
  a.top = static_cast<int>(std::nearbyint((RH - crop) / 2.0));
  a.left = static_cast<int>(std::nearbyint((RW - crop) / 2.0));
  a.sy = static_cast<float>(static_cast<double>(H) / RH);
  a.sx = static_cast<float>(static_cast<double>(W) / RW);
  for (int c = 0; c < 3; ++c) {
    if (!(stdv[c] > 0.f)) return VITB200_E_INVALID_ARG;
    a.mean[c] = mean[c];
    a.inv_std[c] = 1.f / stdv[c];
  }
  int dev = 0;
  if (int st = cuda_status(cudaGetDevice(&dev))) return st;
  int sms = 0;
  if (int st = cuda_status(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)))
    return st;
  const int64_t work = static_cast<int64_t>(B) * crop * crop;
  const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, static_cast<int64_t>(sms) * 8));
  if (int st = launch_kernel(preprocess_kernel, dim3(grid), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), 1, images, out, a))
    return st;
  return cuda_status(cudaGetLastError());
}
