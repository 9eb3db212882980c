/*
 * oracle.h — CPU restatement of OnnxSharp's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA kernels
 * in libonnxsharp_cuda and the timed CPU baseline in bench.py. Only tests/,
 * __graft_entry__.smoke() and bench.py (its CPU-baseline and reference arms)
 * may load it; the product never calls it and has no CPU fallback.
 *
 * Parity pin: the reference is C# and cannot be built in this environment
 * (no dotnet/mono), so this is a restatement, pinned against the known-answer
 * vectors and invariants of the reference's own tests (tests/golden/, see
 * tests/test_oracle.py). Each function names the reference file:line it
 * follows. Arithmetic is plain IEEE binary32 with explicit fmaf() where the
 * reference calls Fma.MultiplyAdd; the library is compiled with
 * -ffp-contract=off so no other operation is fused.
 */
#ifndef ONNXSHARP_ORACLE_H
#define ONNXSHARP_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Tensors/VectorMath.cs:21-43, :70-77 (vector-lane semantics). */
float orc_exp(float x);
float orc_sigmoid(float x);
float orc_silu(float x);
/* y[i] = act(x[i]) over n elements (act: 0 none, 1 SiLU, 2 ReLU, 3 Sigmoid). */
void orc_unary(const float* x, float* y, long n, int act, int threads);

/* GemmKernel.Multiply / MultiplyPacked (Tensors/GemmKernel.cs:131-269, :675-852,
 * micro-kernels :1070-1304, tails :1594-1608, :1645-1792):
 *   acc = row_bias[i] | col_bias[j] | 0;  acc = fmaf(a[i,t], b[t,j], acc), t ascending;
 *   with col_scale: acc from 0, then fmaf(acc, scale[j], col_bias[j]) on full
 *   16-column panels of 12/6/4-row groups, acc*scale[j] + col_bias[j] (two
 *   roundings) on tail columns and leftover rows (mr12: AVX-512 row grouping).
 * b is [k, n] with row pitch ldb. act is applied afterwards (in place). */
void orc_gemm_f32(const float* a, int lda, const float* b, int ldb, int m, int k, int n, const float* row_bias,
                  const float* col_bias, const float* col_scale, int mr12, int act, float* c, int ldc, int threads);

/* Quantizer.MinMax (Tensors/Quantization.cs:109-181): min/max including 0, NaN skipped. */
void orc_minmax(const float* x, long n, float* out_min, float* out_max);

/* DynamicQuantizeMatMul parameters (Ops/QuantizedMatMulOps.cs:146-156):
 * scale = (max-min)/255, 1 if !(scale > 0); zp = clamp((int)rne(-min/scale), 0, 255). */
void orc_dql_params(float mn, float mx, float* scale, int* zero_point);

/* Quantizer.QuantizeToUInt8 (Quantization.cs:68-103): clamp(rne(x*(1/scale)) + zp, 0, 255). */
void orc_quantize_u8(const float* x, long n, float scale, int zero_point, uint8_t* q, int threads);

/* DynamicQuantizeMatMulLayer.Forward (Ops/QuantizedMatMulOps.cs:115-201) with the
 * prepacked path: y = epilogue(sum_t (q[i,t]-zp) * (w[t,j]-w_zp[j])).
 * w is [k, n] int8 (w_signed=1) or uint8; w_zp has n_zp entries (1 or n);
 * w_scale has n_scale entries (1 or n); bias may be NULL. Optional outputs:
 * q_out [m,k] u8, acc_out [m,n] s32, params_out {scale, zp}. */
void orc_dqmm(const float* a, int m, int k, const void* w, int w_signed, const int32_t* w_zp, int n_zp,
              const float* w_scale, int n_scale, const float* bias, int n, int mr12, float* y, uint8_t* q_out,
              int32_t* acc_out, float* params_out, int threads);

/* Exact integer MatMulInteger: acc[i,j] = sum_t (a[i,t]-a_zp) * (w[t,j]-w_zp[j])
 * (Kernels/Int8Gemm.cs:212-238, MultiplyIntegerScalar). */
void orc_matmul_integer(const void* a, int a_signed, int m, int k, int a_zp, const void* w, int w_signed,
                        const int32_t* w_zp, int n_zp, int n, int32_t* acc, int threads);

/* ConvKernels.Im2Col (Kernels/ConvKernels.cs:262-462, :525-654): NCHW, groups,
 * stride, dilation, pads; acc = bias[oc], then fmaf over K = (ic, ky, kx)
 * ascending with padded taps contributing fmaf(w, 0, acc); then act
 * (Ops/DnnOps.cs:493-499). */
void orc_conv2d(const float* x, int N, int C, int H, int W, const float* w, int M, int kh, int kw, int sh, int sw,
                int pt, int pl, int dh, int dw, int group, const float* bias, int act, float* y, int OH, int OW,
                int threads);

/* AttentionLayer.Forward (Ops/AttentionOps.cs:249-351): ComputeBlocks (:464-690)
 * when T > block_min_seq (default 64), else ComputeRows (:353-440).
 * heads_form=1: Q/K/V are [B,T,H*D]; 0: Q [B,H,T,D], K [B,H,D,T], V [B,H,T,D].
 * mask (may be NULL) is [B,1,1|T,T]; mask_rows = 1 or T. out is [B,T,H*D]
 * (out_head_space=0) or [B,H,T,D]. */
void orc_attention(const float* q, const float* k, const float* v, const float* mask, int mask_rows, int B, int T,
                   int H, int D, float scale, int heads_form, int out_head_space, int block_min_seq, float* out,
                   int threads);

/* SoftmaxLayer over the last axis (Ops/DnnOps.cs:2547) -> VectorMath.SoftmaxRow per row. */
void orc_softmax_rows(const float* x, float* y, long rows, int len, int threads);

/* DflLayer.ApplyBlock (Ops/DflOps.cs:167-250): x [B, sides*bins, pixels] ->
 * out [B, sides, pixels] = sum_b b * softmax_b. */
void orc_dfl(const float* x, int B, int sides, int bins, int pixels, float* out, int threads);

/* LayerNormLayer.Forward (Ops/AttnOps.cs:199-358), 16-lane (AVX-512) path. */
void orc_layernorm(const float* x, int outer, int inner, const float* gamma, const float* beta, float eps,
                   float* y, int threads);

/* ImagePreprocessor.Letterbox (Vision/ImagePreprocessor.cs:57-100) with
 * ImageGeometry.Contain (Imaging/AxisMap.cs:97-112), AxisMap.Bilinear
 * (:22-40) and ImageTensor.ToChw (Imaging/ImageTensor.cs:13-170), Divide255
 * normalisation: u8 pixels (bytes_per_pixel 3 or 4, channel c at byte
 * offset bgr ? 2 - c : c) -> dst [3, th, tw], pad 114/255. placement gets
 * {resized_w, resized_h, offset_x, offset_y}. */
void orc_letterbox(const uint8_t* pixels, int width, int height, int row_stride, int bytes_per_pixel, int bgr, int tw,
                   int th, float* dst, int* placement);

#ifdef __cplusplus
}
#endif

#endif
