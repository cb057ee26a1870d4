/* Test infrastructure only: the CPU parity checker for the decode hot path.
 *
 * A plain-C restatement of the reference's CPU algorithm (file:line citations on each
 * function in xq_oracle.c). It is pinned bit-exact against the reference library compiled
 * from its own sources (oracle/_ref) and against the reference's own known-answer tests.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it.
 */
#ifndef XQ_ORACLE_H_
#define XQ_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct xo_matrix {
    int rows;
    int cols;
    int group_size;
    int version; /* 1: (code - zero) * scale, 2: code * scale + zero */
    const uint8_t* packed; /* rows * ceil(cols/2) bytes, even column in the low nibble */
    const float* scales;   /* rows * ceil(cols/group) */
    const float* zeros;    /* rows * ceil(cols/group) */
} xo_matrix;

void xo_set_threads(int threads);
int xo_get_threads(void);

void xo_gemv_w4a16(const xo_matrix* m, const float* x, float* y);
int xo_gemv_w4a16_argmax(const xo_matrix* m, const float* x, float* out_value);
void xo_rmsnorm(const float* x, const float* weight, int n, float eps, float* y);
void xo_head_rmsnorm(float* x, const float* weight, int heads, int head_dim, float eps);
void xo_l2norm_heads(float* x, int heads, int head_dim);
void xo_gated_head_rmsnorm(const float* input, const float* weight, const float* gate, int heads,
                           int head_dim, float eps, float* output);
void xo_rope_partial(float* x, int heads, int head_dim, int rotary_dim, int position, float theta);
void xo_attention_decode(const float* q, const float* k_cache, const float* v_cache, int context,
                         int kv_heads, int q_heads, int head_dim, float* out);
void xo_conv1d_step(const float* mixed, float* state, const float* weight, int channels, int kernel,
                    float* out);
void xo_gated_delta_decode(const float* q, const float* k, const float* v, float beta, float gate,
                           int key_dim, int value_dim, float* state, float* out);
float xo_silu(float x);
float xo_sigmoid(float x);
float xo_softplus(float x);

/* Whole-model restatement (CustomModel: custom_model.cpp:423-1356). */
typedef struct xo_model xo_model;
xo_model* xo_model_load(const char* model_dir, char* error, size_t error_capacity);
void xo_model_free(xo_model* m);
void xo_model_reset(xo_model* m);
int xo_model_prefill(xo_model* m, const int32_t* ids, size_t n, char* error, size_t error_capacity);
int xo_model_decode_one(xo_model* m, int32_t* token, char* error, size_t error_capacity);
int xo_model_hidden_size(const xo_model* m);
int xo_model_layers(const xo_model* m);
int xo_model_position(const xo_model* m);
void xo_model_hidden(const xo_model* m, float* out);
/* Full lm_head logits of the current hidden state (vocab floats). */
void xo_model_logits(const xo_model* m, float* out);
/* Per-layer state for state-level parity checks; returns element count, 0 if absent. */
size_t xo_model_conv_state(const xo_model* m, int layer, float* out);
size_t xo_model_recurrent_state(const xo_model* m, int layer, float* out);
size_t xo_model_kv(const xo_model* m, int layer, float* k_out, float* v_out);

#ifdef __cplusplus
}
#endif

#endif /* XQ_ORACLE_H_ */
