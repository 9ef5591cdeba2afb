#pragma once

/*
 * welvet_c.h -- the welvet.cuda C ABI entry points served by the B200 (sm_100a) library
 * libwelvet_b200.so. Names, argument order and meaning, enum values and the welvet_status
 * layout are those of the reference header include/welvet_c.h, so a program built against
 * the reference links against this library unchanged.
 *
 * Conventions kept from the reference:
 *   - all pointers are host pointers and are copied during the call; nothing is retained
 *     (reference include/welvet_c.h:41-44);
 *   - status codes 0 ok, 1 invalid argument, 2 unsupported, 3 gap, 4 internal
 *     (reference include/welvet_c.h:26-29, include/welvet/status.hpp:8-14);
 *   - DType ids: Float32 1, FP8E4M3 4, FP8E5M2 5, Int8 9, FP4 16 (include/welvet/dtype.hpp:9-44);
 *     other ids return status 2 -- the library never falls back to the host;
 *   - Activation ids -1 Linear, 0 ReLU, 1 SiLU, 2 GELU(tanh), 3 Tanh, 4 Sigmoid, 5 LeakyReLU,
 *     6 ReLU2 (include/welvet/activate.hpp:8-17);
 *   - calls are synchronous; a dense session is not locked (callers serialize its use).
 *
 * The Dense training step (welvet_dense_normalbp_f32) runs on the GPU. The remaining
 * reference symbols (the other layers' NormalBP entry points, the other layer kinds and the
 * WMN1 model-session training family) are exported with their reference signatures and
 * return status 3 ("gap") from this library.
 */

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WELVET_API __attribute__((visibility("default")))

/* reference include/welvet_c.h:26-29 */
typedef struct welvet_status {
  int32_t code;
  char message[256];
} welvet_status;

/* reference include/welvet_c.h:31 -- opaque resident Dense session */
typedef struct welvet_dense_session welvet_dense_session;

/* reference include/welvet_c.h:33-36. welvet_version returns the reference ABI level ("0.79");
 * welvet_runtime_identity "cuda:<name>:idx=<i>:sm=<major>.<minor>:mem=<bytes>". */
WELVET_API const char* welvet_version(void);
WELVET_API const char* welvet_runtime_identity(void);

/* reference include/welvet_c.h:37-38. Init selects the library device: the device current
 * in the calling thread on first use (0 unless the application chose one) or
 * $WELVET_B200_DEVICE. */
WELVET_API welvet_status welvet_cuda_init(void);
WELVET_API int32_t welvet_cuda_available(void);

/* reference include/welvet_c.h:64-67 -- one-shot Dense forward: quantize W (out x in,
 * row-major float32) with `dtype`, run batch rows of x through y = act(W x + bias).
 * pre/post are [batch*out]. `backend` is ignored, as in the reference (c_abi.cpp:96). */
WELVET_API welvet_status welvet_dense_forward_f32(
    int32_t batch, int32_t in, int32_t out, int32_t act, int32_t dtype, int32_t backend,
    const float* W_init, const double* bias, size_t bias_len, const float* x, float* pre,
    float* post);

/* reference include/welvet_c.h:69-78 (src/interop/c_abi.cpp:119-184) --
 * one Dense training step on the GPU: quantize W_init, forward x (pre/post [batch*out]), take
 * the output gradient from grad_or_target (use_target != 0: MSE against it as a target, *loss
 * = mean squared error, else *loss = 0), backward (dX [batch*in], dW [out*in]), SGD
 * W <- W - lr*dW on the quantized store when lr != 0, and W_after [out*in] = the store's
 * decoded weights. Status 1 "invalid argument" for a null pointer or a non-positive size,
 * 1 "bad dtype N" outside 0..33, 2 for dtypes off the GPU path. */
WELVET_API welvet_status welvet_dense_normalbp_f32(
    int32_t batch, int32_t in, int32_t out, int32_t act, int32_t dtype, int32_t backend,
    const float* W_init, const double* bias, size_t bias_len, const float* x,
    const float* grad_or_target, int32_t use_target, double lr, float* pre, float* post,
    float* dX, float* dW, float* W_after, double* loss);

/* reference include/welvet_c.h:81-86 -- resident session: mount once (quantize on the GPU,
 * keep the packed codes resident), execute many (H2D x, fused dequant GEMV + bias/act,
 * D2H pre/post, synchronize). */
WELVET_API welvet_status welvet_dense_mount(int32_t batch, int32_t in, int32_t out, int32_t act,
                                            int32_t dtype, const float* W_init, const double* bias,
                                            size_t bias_len, welvet_dense_session** sess_out);
WELVET_API welvet_status welvet_dense_execute(welvet_dense_session* sess, const float* x, float* pre,
                                              float* post);
WELVET_API void welvet_dense_release(welvet_dense_session* sess);

/* reference include/welvet_c.h:89-92 -- RMSNorm forward (gamma quantized with dtype, eps <= 0
 * -> 1e-6). pre = x * inv_rms, post = pre * gamma; [batch*seq*dim]. */
WELVET_API welvet_status welvet_rmsnorm_forward_f32(int32_t batch, int32_t seq, int32_t dim,
                                                    double eps, int32_t dtype, int32_t backend,
                                                    const float* gamma, const float* x, float* pre,
                                                    float* post);

/* reference include/welvet_c.h:132-135 -- SwiGLU forward: pre = h = SiLU(Gate x) * (Up x)
 * [batch*seq*intermediate], post = Down h [batch*seq*input]. Gate/Up are
 * [intermediate x input], Down [input x intermediate]; one dtype for all three. */
WELVET_API welvet_status welvet_swiglu_forward_f32(
    int32_t batch, int32_t seq, int32_t input_dim, int32_t intermediate_dim, int32_t dtype,
    int32_t backend, const float* Gate, const float* Up, const float* Down, const float* x,
    float* pre, float* post);

/* reference include/welvet_c.h:165-169 -- MHA ModeSelf forward: Q/K/V projections, attention
 * core (fp64, the reference's KV-ring semantics), O projection. pre = attention output
 * [batch*seq*q_dim], post = O(attn) [batch*seq*d_model]. mask/pos are the reference's
 * MaskKind / PosKind values (include/welvet/mha.hpp:12-27). */
WELVET_API welvet_status welvet_mha_forward_f32(
    int32_t batch, int32_t seq, int32_t d_model, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t max_seq_len, int32_t mask, int32_t pos, int32_t dtype,
    int32_t backend, const float* Q, const float* K, const float* V, const float* O, const float* x,
    float* pre, float* post);

/* reference include/welvet_c.h:39-40 -- the gaps census: this library counts its own
 * status-3 entry points. */
WELVET_API int32_t welvet_gaps_count(void);
WELVET_API int32_t welvet_gaps_done(void);

/* reference include/welvet_c.h:45-61 -- persistent model sessions and their blobs. */
typedef struct welvet_model_session welvet_model_session;
typedef struct welvet_cuda_blob { uint8_t* data; size_t size; } welvet_cuda_blob;
WELVET_API int32_t welvet_model_abi_version(void);
WELVET_API void welvet_cuda_blob_free(welvet_cuda_blob*);
/* reference include/welvet_c.h:48-49 and the release of model_session.cpp -- a WMN1 model
 * descriptor (Stack or Grid root of Dense / RMSNorm / SwiGLU / MHA children, weights from its
 * store section) mounted on the GPU; forward takes and returns tensor records (int32 rank,
 * int32 dims, float32 data), the output blob freed with welvet_cuda_blob_free. Other roots
 * and child kinds: status 3. The other welvet_model_* entry points (training) are gaps. */
WELVET_API welvet_status welvet_model_mount(const uint8_t* descriptor, size_t size, welvet_model_session** out);
WELVET_API welvet_status welvet_model_forward(welvet_model_session* s, const uint8_t* input, size_t size,
                                              welvet_cuda_blob* out);
WELVET_API void welvet_model_release(welvet_model_session* s);

#ifdef __cplusplus
}
#endif
