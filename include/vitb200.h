/*
 * vitb200.h — C ABI of the B200-native ViT-B/16 engine (libvitb200.so).
 *
 * Every entry point takes plain device pointers, element counts and a
 * cudaStream_t (passed as void* so this header needs no CUDA include), launches
 * asynchronously on that stream and returns an int status:
 *     0                         success
 *     > 0                       a cudaError_t raised by a launch or a runtime call
 *     < 0                       a VITB200_E_* code below (nothing was launched)
 * Nothing here allocates device memory except where a function says so: scratch
 * space is a caller-provided workspace whose size a *_workspace_bytes() query
 * returns. All launches go to the given stream with no host synchronisation, so
 * every entry point can be captured in a CUDA graph once the library has been
 * initialised on the device (vitb200_init, or any earlier call).
 *
 * All tensors are fp32, row-major and contiguous unless a leading dimension is
 * given. A "TF32 pair" is a [2][rows][cols] buffer: plane 0 holds
 * hi = round_tf32(x), plane 1 holds lo = round_tf32(x - hi); the GEMM core
 * consumes operands in this form (three tcgen05 TF32 products per K step:
 * hi*hi + hi*lo + lo*hi).
 *
 * The reference interface each function replaces is cited as path:line inside
 * the reference project AhmadSaeedZaidi/ViT-Engine-CUDA.
 */
#ifndef VITB200_H
#define VITB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default) /* the library builds with hidden defaults */
#endif

/* ---- status codes ------------------------------------------------------ */
#define VITB200_OK 0
#define VITB200_E_INVALID_ARG (-1)    /* null pointer, negative or inconsistent size */
#define VITB200_E_UNSUPPORTED (-2)    /* a shape this build does not implement        */
#define VITB200_E_WORKSPACE (-3)      /* workspace smaller than *_workspace_bytes()   */
#define VITB200_E_DEVICE_TIMEOUT (-4) /* a kernel gave up on a bounded wait           */
#define VITB200_E_NO_TMA (-5)         /* cuTensorMapEncodeTiled unavailable/failed    */
#define VITB200_E_ALIGNMENT (-6)      /* pointer or stride not 16-byte aligned        */

/* GEMM epilogues (vitb200_gemm). Y = X * W^T computed in TF32x3, then: */
#define VITB200_EPI_NONE 0      /* Y = acc                                          */
#define VITB200_EPI_BIAS 1      /* Y = acc + bias                                   */
#define VITB200_EPI_BIAS_GELU 2 /* Y = gelu_erf(acc + bias)                         */
#define VITB200_EPI_BIAS_RESID 3/* Y = residual + acc + bias (residual may alias Y) */

/* ---- library / device management -------------------------------------- */

/* Library version as 10000*major + 100*minor + patch. */
int vitb200_version(void);

/* Human-readable text for a status code. Never returns NULL. */
const char* vitb200_status_string(int status);

/* Prepares the current device: resolves the device error word, raises the
 * dynamic shared-memory limits of the kernels. Idempotent; call it (or any
 * other entry point) once per device before capturing a CUDA graph. */
int vitb200_init(void);

/* Reads (and optionally clears) the current device's error word, written by
 * kernels whose bounded waits ran out. Synchronises the device. *code is 0
 * when no kernel reported an error. */
int vitb200_device_error(int* code, int clear);

/* Failure-reporting check: launches a kernel whose bounded wait is never
 * satisfied (kind 0: the GEMM / attention pipeline wait, which reports code
 * 1; kind 1: a split-K owner's cluster-scope wait, code 7). After the wait
 * limit (1 s) it records the code in the device error word and returns; the
 * context stays usable. No counterpart in the reference (its kernels have no
 * waits). */
int vitb200_check_wait_timeout(int kind, void* stream);

/* Number of streaming multiprocessors the launch heuristics use. */
int vitb200_num_sms(void);

/* Kernel launches this library has issued in this process (all devices, all
 * streams; a CUDA-graph replay issues none). For benchmarks and tests. */
uint64_t vitb200_launch_count(void);

/* GEMM tile configuration: 0 = automatic (default); 1..15 force one of the
 * compiled configurations. On TF32 pairs: 1 = 128x128 tiles, 2 stages of K=32;
 * 2 = 128x128, 5 stages of K=16; 3 = 128x64, 3 stages of K=32; 4 = as 1 with K
 * chunks of 64; 5 = 128x256, 3 stages of K=16; 6 = 256x256 on a CTA pair, 2
 * stages of K=32; 7 = 256x256 pair, 5 stages of K=16; 8 = as 7 with K chunks of
 * 256. On FP16 splits (vitb200_gemm_f16 and the model's F16 path): 9 = 256x256
 * pair, 2 stages of K=64; 10 = 128x128, 2 stages of K=64; 11 = 128x64, 3
 * stages of K=64; 12 = 256x256 pair, 4 stages of K=32; 13, 14 = as 9, 10 with
 * two W planes (cross products folded in by tcgen05.mma's scale-input-d, K
 * chunks of 64); 15 = as 9 with K chunks of 256. A forced configuration
 * of the other operand kind is ignored. All accumulate K in chunks (128 unless
 * stated) on the tensor core and sum the chunks in FP32 registers. Returns the
 * previous setting. For tuning and tests; process-wide. */
int vitb200_set_gemm_variant(int variant);

/* Split-K of small single-CTA GEMM launches (on by default). When the output
 * tile grid fills at most half the SMs (e.g. the block GEMMs of a batch-1
 * forward, M = 197 rows), the launch splits K into d <= 8 equal parts over a
 * thread-block cluster of d CTAs per tile; each CTA keeps its fp32 partial
 * tile in its shared memory, and the tile's 32 x 32 slabs are shared out among
 * the cluster's CTAs, each adding the partials of its slabs in split order
 * over distributed shared memory (deterministic) and writing them. An image's logits are bitwise identical in any batch of at least 7
 * images at 224x224 (CTA-pair tiles from 1024 token rows, no split); with
 * split-K off also among batches of up to 5 images; otherwise they agree to
 * FP32 rounding. No counterpart in the reference (one CTA per 32x32 output
 * tile there). Affects launches made after the call (a captured CUDA graph
 * keeps the setting it was captured with). Returns the previous setting;
 * process-wide. */
int vitb200_set_split_k(int enable);

/* Forces the K split of later small single-CTA GEMM launches (those split-K
 * applies to) to ksplit CTAs per tile wherever that split fits (ksplit divides
 * the K blocks, the CTAs fit in one wave and the clusters are co-resident);
 * 0 restores the automatic choice, values outside 0..8 are ignored. No effect
 * while split-K is off. Returns the previous setting. For tuning and tests;
 * process-wide. */
int vitb200_set_gemm_split(int ksplit);

/* The tile configuration (*variant, as in vitb200_set_gemm_variant) and the K
 * split (*ksplit, 1 = none) that a GEMM of M x K by K x N (f16 = 1: FP16-split
 * operands, 0: TF32 pairs) launched now on the current device would use.
 * Either output may be NULL. For diagnostics and tests. */
int vitb200_gemm_plan(int64_t M, int K, int N, int f16, int* variant, int* ksplit);

/* ---- TF32 split -------------------------------------------------------- */

/* Writes the TF32 pair of x[rows][cols] (row stride ldx floats) into
 * pair[2][rows][ldp]; columns cols..ldp-1 are zero-filled (ldp >= cols,
 * ldp % 4 == 0). Weight pre-splitting and the per-op GEMM wrappers use it.
 * No reference counterpart: the reference splits inside its opt-in CuTe GEMM
 * (csrc/kernels/gemm_cute_tf32.cu:104-115). */
int vitb200_split_tf32(const float* x, int64_t rows, int cols, int64_t ldx,
                       float* pair, int ldp, void* stream);

/* Image preprocessing, the step before the forward in the reference
 * (vit_cuda/model.py:180-188: torchvision Resize(resize_short) ->
 * CenterCrop(crop) -> ToTensor -> Normalize(mean, std)). images: B equal-size
 * 8-bit RGB images, HWC, image_stride bytes apart (>= H*W*3), on the device.
 * The shorter side is resized to resize_short (the longer to
 * floor(resize_short * long / short)) with antialiased bilinear resampling in
 * fp32, the centred crop x crop window kept (offsets rounded half to even),
 * and out[B][3][crop][crop] = (x / 255 - mean[c]) / std[c]; mean and std are
 * 3-element host arrays. VITB200_E_UNSUPPORTED when the resized image is
 * smaller than the crop (torchvision would pad). */
int vitb200_preprocess(const uint8_t* images, int B, int H, int W,
                       int64_t image_stride, int resize_short, int crop,
                       const float* mean, const float* std, float* out,
                       void* stream);

/* ---- per-op entry points (reference: csrc/bindings/binding.cpp:5-23) --- */

/* LayerNorm over the last dim E of x[rows][E]: biased variance, affine.
 * Replaces launch_layernorm (csrc/kernels/layernorm.cu:67-80) behind
 * layernorm_forward (csrc/ops/layernorm_wrapper.cpp:16-45). Any E % 4 == 0. */
int vitb200_layernorm(const float* x, const float* gamma, const float* beta,
                      float* y, int64_t rows, int E, float eps, void* stream);

/* GEMM Y[M][N] = epilogue(X[M][K] * W[N][K]^T) in TF32x3 on tcgen05.
 * Replaces launch_gemm / launch_gemm_bias / launch_gemm_gelu
 * (csrc/include/gemm_kernels.h:8-38, csrc/kernels/gemm.cu:98-143) and the
 * C-ABI probe run_gemm (tools/gemm_probe.cu:4-16). M, K, N >= 0, any value.
 * bias: [N] (required for the BIAS* epilogues); residual: [M][N] (BIAS_RESID).
 * The workspace holds the TF32 pairs of X and W. */
size_t vitb200_gemm_workspace_bytes(int64_t M, int K, int N);
int vitb200_gemm(const float* X, const float* W, const float* bias,
                 const float* residual, float* Y, int64_t M, int K, int N,
                 int epilogue, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Allocation-free variant of vitb200_gemm, for callers that cannot allocate
 * device memory: a C or ctypes host program with no device allocator of its
 * own, a host whose device memory is owned by another framework's pool, or a
 * request path that cannot afford cudaMalloc's device-wide synchronisation.
 * Same arguments (minus the workspace) and the same results as vitb200_gemm;
 * the TF32 pairs of X and W live in a fixed 16 MiB array inside the library
 * (resident on every GPU that loads it until the process exits). Limit:
 * 2*M*Kp rounded up to 64, plus 2*N*Kp, at most 4,194,304 floats (Kp = K rounded
 * up to 4; e.g. M = N = K = 1024); larger problems return VITB200_E_WORKSPACE
 * without launching. Calls share that array: calls whose GPU work can overlap
 * (unordered streams, concurrent host threads) race; calls on one stream are
 * safe. The first call on a device looks up the array's device address; make
 * it before any stream capture. That address is kept for the life of the
 * process, so do not call this again on a device after cudaDeviceReset.
 * Allocates nothing. It has no counterpart in the reference. */
int vitb200_gemm_noalloc(const float* X, const float* W, const float* bias,
                         const float* residual, float* Y, int64_t M, int K, int N,
                         int epilogue, void* stream);

/* GEMM core on pre-split operands: a_pair [2][M][Kp], w_pair [2][N][Kp]
 * (Kp % 4 == 0, zero padded past K). Writes fp32 Y (ldy) and/or the TF32 pair
 * of the result (y_pair, [2][M][N]) — either may be NULL, not both. */
int vitb200_gemm_pairs(const float* a_pair, const float* w_pair, const float* bias,
                       const float* residual, float* Y, int64_t ldy, float* y_pair,
                       int64_t M, int Kp, int N, int epilogue, void* stream);

/* FP16 split of x[rows][cols] (row stride ldx) times `scale`, written as
 * nplanes (2 or 3) planes of planes[nplanes][rows][ldp] fp16 (ldp % 8 == 0,
 * zero past cols): hi = fp16(x*scale), lo = fp16((x*scale - hi) * 2^11) and,
 * with nplanes == 3, hi * 2^11 (the third plane a GEMM's W operand needs).
 * Scaled magnitudes must stay below 32768 (below 16 with nplanes == 3); a
 * larger or non-finite value sets the device error (vitb200_device_error)
 * instead of failing silently.
 * No reference counterpart: operand preparation of vitb200_gemm_f16. */
int vitb200_split_f16(const float* x, int64_t rows, int cols, int64_t ldx, float scale,
                      uint16_t* planes, int64_t ldp, int nplanes, void* stream);

/* GEMM core on FP16-split operands (the three-product FP16 emulation of an
 * FP32 GEMM): a_planes [2][M][Kp] from vitb200_split_f16 with scale 1 and
 * nplanes 2, w_planes [3][N][Kp] from vitb200_split_f16 with scale s and
 * nplanes 3, acc_scale = 2^-11 / s (Kp % 8 == 0, zero padded past K).
 * Writes fp32 Y (ldy) and/or the FP16 split of the result (y_h16,
 * [2][M][N]) — either may be NULL, not both. Accuracy matches
 * vitb200_gemm_pairs (TF32x3); throughput is twice the TF32 rate. No
 * reference counterpart: the reference's GEMMs are FP32 SIMT or TF32x3
 * (csrc/kernels/gemm.cu:12-96, csrc/kernels/gemm_cute_tf32.cu:53-168). */
int vitb200_gemm_f16(const uint16_t* a_planes, const uint16_t* w_planes, float acc_scale,
                     const float* bias, const float* residual, float* Y, int64_t ldy,
                     uint16_t* y_h16, int64_t M, int Kp, int N, int epilogue, void* stream);

/* QKV projection: X[M][E] * W[3E][E]^T + b, written as three contiguous
 * [M][E] planes q, k, v of qkv_out[3][M][E]. Replaces qkv_kernel_launcher
 * (csrc/kernels/qkv.cu:5-16) plus the three .contiguous() copies of
 * csrc/ops/qkv_wrapper.cpp:49-52. */
size_t vitb200_qkv_workspace_bytes(int64_t M, int E);
int vitb200_qkv(const float* X, const float* W, const float* b, float* qkv_out,
                int64_t M, int E, void* workspace, size_t workspace_bytes,
                void* stream);

/* MLP: H = gelu_erf(X W1^T + b1), O = H W2^T + b2 (X[M][E], H[M][E4]).
 * Replaces mlp_forward_cuda (csrc/kernels/mlp.cu:5-20). */
size_t vitb200_mlp_workspace_bytes(int64_t M, int E, int E4);
int vitb200_mlp(const float* X, const float* W1, const float* b1,
                const float* W2, const float* b2, float* H, float* O,
                int64_t M, int E, int E4, void* workspace,
                size_t workspace_bytes, void* stream);

/* Non-causal multi-head attention softmax(Q K^T * scale) V over
 * q/k/v[B][T][heads*64] (row strides ldq/ldk/ldv floats), head h in columns
 * h*64..h*64+63, on the tensor cores in TF32x3. Writes o[B][T][heads*64] (row
 * stride ldo, 16-byte aligned). The workspace holds the TF32 pairs of q, k, v.
 * Replaces flash_attn_2_forward_cuda (csrc/kernels/attention.cu:208-226). */
size_t vitb200_attention_workspace_bytes(int B, int T, int heads);
int vitb200_attention(const float* q, const float* k, const float* v, float* o,
                      int B, int T, int heads, int64_t ldq, int64_t ldk,
                      int64_t ldv, int64_t ldo, float scale, void* workspace,
                      size_t workspace_bytes, void* stream);

/* The same attention with FP16-split operands (three FP16 tensor-core
 * products per multiply, FP32 accuracy; the form the model's block path
 * uses). k and v are multiplied by k_scale and v_scale (powers of two, undone
 * exactly; 1 is fine) before the split; |q|, |k * k_scale| and |v * v_scale|
 * must stay below 32768 (larger values set the
 * device error). The workspace holds the FP16 splits of q, k and V^T. No
 * reference counterpart beyond flash_attn_2_forward_cuda's semantics. */
size_t vitb200_attention_f16_workspace_bytes(int B, int T, int heads);
int vitb200_attention_f16(const float* q, const float* k, const float* v, float* o,
                          int B, int T, int heads, int64_t ldq, int64_t ldk,
                          int64_t ldv, int64_t ldo, float scale, float k_scale,
                          float v_scale, void* workspace, size_t workspace_bytes,
                          void* stream);

/* Patch embedding as im2col + TF32x3 GEMM: img[B][C][H][W] (16x16 patches,
 * vector order (c, py, px)), weights [E][C*256] -> out[B][P][E] (+ bias when
 * bias != NULL). Replaces launch_patch_embed (csrc/kernels/patch_embed.cu:100-110)
 * and the bias add of csrc/ops/patch_embed_wrapper.cpp:46-48; H and W are
 * runtime values (multiples of 16). */
size_t vitb200_patch_embed_workspace_bytes(int B, int C, int H, int W, int E);
int vitb200_patch_embed(const float* img, const float* weights, const float* bias,
                        float* out, int B, int C, int H, int W, int E,
                        void* workspace, size_t workspace_bytes, void* stream);

/* out[b][0] = cls[b] + pos[0]; out[b][1+p] = patches[b][p] + pos[1+p] with
 * cls[B][E], pos[P+1][E]. Replaces launch_pos_encoding
 * (csrc/kernels/pos_encoding.cu:30-41); P is a runtime value. */
int vitb200_pos_encoding(const float* patches, const float* cls, const float* pos,
                         float* out, int B, int P, int E, void* stream);

/* logits[B][C] = X[b][0][:] . W[c][:] + bias[c] for X[B][T][E] (CLS row only),
 * in TF32x3. Replaces launch_classifier (csrc/kernels/classifier.cu:68-80). */
size_t vitb200_classifier_workspace_bytes(int B, int E, int C);
int vitb200_classifier(const float* X, const float* W, const float* bias,
                       float* logits, int B, int T, int E, int C, void* workspace,
                       size_t workspace_bytes, void* stream);

/* ---- whole-model forward (reference: vit_cuda/model.py:93-126) --------- */

typedef struct vitb200_block_params {
    const float* norm1_w;     /* [768]                         */
    const float* norm1_b;     /* [768]                         */
    const float* qkv_w_pair;  /* TF32 pair of [2304][768]      */
    const float* qkv_b;       /* [2304]                        */
    const float* proj_w_pair; /* TF32 pair of [768][768]       */
    const float* proj_b;      /* [768]                         */
    const float* norm2_w;     /* [768]                         */
    const float* norm2_b;     /* [768]                         */
    const float* fc1_w_pair;  /* TF32 pair of [3072][768]      */
    const float* fc1_b;       /* [3072]                        */
    const float* fc2_w_pair;  /* TF32 pair of [768][3072]      */
    const float* fc2_b;       /* [768]                         */
    /* Optional FP16-split weights (vitb200_split_f16 with 3 planes and scale
     * s; acc_scale = 2^-11 / s). A GEMM whose *_w_f16 is non-NULL runs on the
     * FP16 path (its *_w_pair may then be NULL) and the kernel producing its
     * input writes the FP16 split instead of the TF32 pair. The caller
     * guarantees that input's magnitudes stay below 32768 (a LayerNorm
     * output is bounded by sqrt(E-1)*max|gamma| + max|beta|, a linear map of
     * it by that times the weight rows' absolute sums); values beyond that
     * set the device error. */
    const uint16_t* qkv_w_f16;  float qkv_acc_scale;
    const uint16_t* proj_w_f16; float proj_acc_scale;
    const uint16_t* fc1_w_f16;  float fc1_acc_scale;
    const uint16_t* fc2_w_f16;  float fc2_acc_scale;
    /* attn_f16 != 0: the attention runs on FP16 splits (as
     * vitb200_attention_f16), its q, k, v written by the QKV GEMM multiplied by
     * q_scale, k_scale, v_scale (powers of two). The caller guarantees
     * |q * q_scale|, |k * k_scale| and |v * v_scale| < 32768 (bounds as
     * above). 0: TF32 pairs. */
    int attn_f16;
    float q_scale, k_scale, v_scale;
    /* LayerNorm folded into the GEMM it feeds (used when
     * vitb200_vit_params.ln_fold != 0; may be NULL otherwise): the FP16
     * planes of W * diag(gamma) (scale s, *_acc_scale = 2^-11 / s), c[n] =
     * sum_k W[n][k] gamma[k] and d[n] = sum_k W[n][k] beta[k] + b[n], for qkv
     * with norm1 and fc1 with norm2. */
    const uint16_t* ln_qkv_w_f16; float ln_qkv_acc_scale;
    const float* ln_qkv_c;
    const float* ln_qkv_d;
    const uint16_t* ln_fc1_w_f16; float ln_fc1_acc_scale;
    const float* ln_fc1_c;
    const float* ln_fc1_d;
} vitb200_block_params;

typedef struct vitb200_vit_params {
    int depth;          /* 12 for ViT-B/16                                */
    int embed_dim;      /* 768 (the only value this build implements)    */
    int num_heads;      /* 12                                             */
    int mlp_dim;        /* 3072                                           */
    int patch;          /* 16                                             */
    int in_chans;       /* 3                                              */
    int img_h, img_w;   /* 224x224 (T=197) or 384x384 (T=577), any /16    */
    int num_classes;    /* 1000                                           */
    float ln_eps;       /* 1e-6                                           */
    float attn_scale;   /* 0.125                                          */
    const float* patch_w_pair; /* TF32 pair of [768][in_chans*256], or NULL with patch_w_f16 */
    const float* patch_b;      /* [768]                                   */
    const float* cls_token;    /* [768]                                   */
    const float* pos_embed;    /* [T][768]                                */
    const vitb200_block_params* blocks; /* host array of `depth` entries  */
    const float* norm_w;       /* [768]                                   */
    const float* norm_b;       /* [768]                                   */
    const float* head_w_pair;  /* TF32 pair of [num_classes][768]         */
    const float* head_b;       /* [num_classes]                           */
    /* Patch GEMM on FP16 splits instead of the TF32 pair (either may be
     * NULL, not both; patch_w_f16 wins): the planes [3][768][in_chans*256]
     * (hi, lo*2^11, hi*2^11) of the weight times a power of two s, and
     * patch_acc_scale = 2^-11 / s. The pixels are then split to FP16 by the
     * im2col kernel, so their magnitudes must stay below 32768 (normalised
     * or 0-255 images do); a larger or non-finite pixel sets the device error
     * (code 6, vitb200_device_error) instead of failing silently. */
    const uint16_t* patch_w_f16;
    float patch_acc_scale;
    /* ln_fold != 0 (every block's ln_* fields set, all four block GEMMs on
     * FP16 splits): in launches of fewer than 1024 token rows (up to 5 images
     * at 224x224) the LayerNorms before qkv and fc1 run inside those GEMMs.
     * The residual GEMM before each writes, besides x, the FP16 split of x
     * and per-row statistics over 32-column slabs; the next GEMM multiplies
     * that split by W * diag(gamma) and its epilogue applies
     * rstd * (acc - mean * c) + d. The residual stream's magnitudes must then
     * stay below 32768 (device error 6 otherwise). Replaces 23 of the 24
     * LayerNorm launches of a ViT-B/16 forward; larger launches keep the
     * LayerNorm kernel (faster there). */
    int ln_fold;
} vitb200_vit_params;

/* Workspace needed by vitb200_vit_forward / _features for `batch` images. */
size_t vitb200_vit_workspace_bytes(const vitb200_vit_params* p, int batch);

/* Full ViT forward: img[batch][in_chans][img_h][img_w] -> logits[batch][C].
 * Replaces ViTCUDA._forward_impl (vit_cuda/model.py:101-126). */
int vitb200_vit_forward(const vitb200_vit_params* p, const float* img,
                        float* logits, int batch, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Same forward stopped after the final LayerNorm of the CLS token:
 * features[batch][768]. The reference's evaluation scripts take these CLS
 * features (scripts/eval_imagenette.py:49-69). */
int vitb200_vit_forward_features(const vitb200_vit_params* p, const float* img,
                                 float* features, int batch, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* The forward in three pieces, the same kernels the full forward chains, for
 * sub-step comparison as the reference's scripts/layerwise_compare.py:141-257
 * does it (embedding, each block, final norm + head). All take the workspace
 * of vitb200_vit_workspace_bytes(p, batch); x is the caller's [batch*T][768]
 * residual stream.
 *   embed: x = [cls + pos[0]; patch_embed(img) + pos[1:]]
 *          (vit_cuda/model.py:103-118)
 *   block: one encoder block `layer` in place on x (vit_cuda/model.py:39-60)
 *   head:  final LayerNorm of the CLS rows -> features (optional) and
 *          logits (optional) (vit_cuda/model.py:123-124) */
int vitb200_vit_embed(const vitb200_vit_params* p, const float* img, float* x,
                      int batch, void* workspace, size_t workspace_bytes,
                      void* stream);
int vitb200_vit_block(const vitb200_vit_params* p, int layer, float* x, int batch,
                      void* workspace, size_t workspace_bytes, void* stream);
int vitb200_vit_head(const vitb200_vit_params* p, const float* x, float* logits,
                     float* features, int batch, void* workspace,
                     size_t workspace_bytes, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* VITB200_H */
