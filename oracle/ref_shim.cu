// C entry points over the reference project's own CUDA launchers — TEST
// INFRASTRUCTURE ONLY (a checker; nothing in vit_cuda links or calls it).
//
// oracle/Makefile compiles this file together with the reference's kernel
// sources, where they lie in the reference tree (csrc/kernels/*.cu), into
// oracle/_ref/libvitref.so for sm_100a with the reference's own flags
// (-O3 -use_fast_math, CMakeLists.txt:52-59). The declarations below restate
// the launcher signatures the reference exports (csrc/include/gemm_kernels.h:8-38
// and the forward declarations of csrc/ops/*_wrapper.cpp); each wrapper
// returns cudaGetLastError() like the reference's probe tools/gemm_probe.cu:4-16.
//
// The reference kernels hardcode E=768 (attention, layernorm), 224x224 images
// (patch_embed) and 197 tokens (pos_encoding, classifier); callers must stay
// inside those shapes, and the GEMMs need K and N multiples of 4.
#include <cuda_runtime.h>

void launch_layernorm(const float* X, const float* gamma, const float* beta, float* Y, int B,
                      int N, float eps, cudaStream_t stream);
void launch_gemm_bias(const float* X, const float* W, const float* B, float* Y, int M, int K,
                      int N_out, cudaStream_t stream);
void launch_gemm(const float* X, const float* W, float* Y, int M, int K, int N_out,
                 cudaStream_t stream);
void launch_gemm_gelu(const float* X, const float* W, const float* B, float* Y, int M, int K,
                      int N_out, cudaStream_t stream);
void flash_attn_2_forward_cuda(const float* Q, const float* K, const float* V, float* O, int B,
                               int N, float scale, cudaStream_t stream);
void launch_patch_embed(float* img, float* weights, float* out, int B, cudaStream_t stream);
void launch_pos_encoding(float* patches, float* cls_token, float* pos_embed, float* out,
                         int batch_size, cudaStream_t stream);
void launch_classifier(const float* X, const float* W, const float* bias, float* Y, int B,
                       int num_classes, cudaStream_t stream);
void mlp_forward_cuda(const float* X, const float* W1, const float* B1, const float* W2,
                      const float* B2, float* H, float* O, int M, int E, int E_expand,
                      cudaStream_t stream);

static int last() { return static_cast<int>(cudaGetLastError()); }

extern "C" {

int ref_layernorm(const float* X, const float* g, const float* b, float* Y, int B, int N,
                  float eps, void* s) {
  launch_layernorm(X, g, b, Y, B, N, eps, static_cast<cudaStream_t>(s));
  return last();
}

int ref_gemm(const float* X, const float* W, const float* bias, float* Y, int M, int K, int N,
             int mode, void* s) {
  cudaStream_t st = static_cast<cudaStream_t>(s);
  if (mode == 2)
    launch_gemm_gelu(X, W, bias, Y, M, K, N, st);
  else if (mode == 1)
    launch_gemm_bias(X, W, bias, Y, M, K, N, st);
  else
    launch_gemm(X, W, Y, M, K, N, st);
  return last();
}

int ref_attention(const float* Q, const float* K, const float* V, float* O, int B, int N,
                  float scale, void* s) {
  flash_attn_2_forward_cuda(Q, K, V, O, B, N, scale, static_cast<cudaStream_t>(s));
  return last();
}

int ref_patch_embed(float* img, float* w, float* out, int B, void* s) {
  launch_patch_embed(img, w, out, B, static_cast<cudaStream_t>(s));
  return last();
}

int ref_pos_encoding(float* patches, float* cls, float* pos, float* out, int B, void* s) {
  launch_pos_encoding(patches, cls, pos, out, B, static_cast<cudaStream_t>(s));
  return last();
}

int ref_classifier(const float* X, const float* W, const float* bias, float* Y, int B, int C,
                   void* s) {
  launch_classifier(X, W, bias, Y, B, C, static_cast<cudaStream_t>(s));
  return last();
}

int ref_mlp(const float* X, const float* W1, const float* B1, const float* W2, const float* B2,
            float* H, float* O, int M, int E, int E4, void* s) {
  mlp_forward_cuda(X, W1, B1, W2, B2, H, O, M, E, E4, static_cast<cudaStream_t>(s));
  return last();
}

}  // extern "C"
