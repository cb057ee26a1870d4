/* A plain C host of libxqwen35.so, compiled against include/xqwen35.h only: the call sequence
 * and checks of the reference's runtime test (customlib/tests/runtime_correctness/
 * test_runtime.cpp:148-211) on the tiny model in argv[1]. Prints the hidden state after prefill,
 * the xq_decode_one token, the xq_generate tokens and the hidden state after them, one per line,
 * then "ok". Any failed check prints "FAIL <line>" and exits 1. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "xqwen35.h"

#define CHECK(c)                                  \
    do {                                          \
        if (!(c)) {                               \
            printf("FAIL %d: %s\n", __LINE__, #c); \
            return 1;                             \
        }                                         \
    } while (0)

static int print_hidden(xq_session* s, const char* tag) {
    float h[64];
    size_t n = 0;
    if (xq_get_hidden_state(s, h, 64, &n) != XQ_OK || n == 0 || n > 64) return 0;
    printf("%s", tag);
    for (size_t i = 0; i < n; ++i) printf(" %.9g", h[i]);
    printf("\n");
    return 1;
}

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    xq_options options;
    memset(&options, 0, sizeof options);
    options.struct_size = sizeof options;
    options.backend = "cpu";
    options.threads = 1;
    options.quant_bits = 4;
    options.group_size = 4;
    options.max_context_tokens = 16;
    options.enable_autotune = 0;
    options.use_mnn_fallback = 0;

    xq_session* session = NULL;
    CHECK(xq_create(argv[1], &options, &session) == XQ_OK);
    CHECK(session != NULL);

    int32_t prompt[3] = {1, 2, 3};
    xq_metrics metrics;
    memset(&metrics, 0, sizeof metrics);
    metrics.struct_size = sizeof metrics;
    CHECK(xq_prefill(session, prompt, 3, &metrics) == XQ_OK);
    CHECK(metrics.prompt_tokens == 3);
    CHECK(print_hidden(session, "hidden_prefill"));

    static char trace[32768];
    CHECK(xq_get_kernel_trace_json(session, trace, sizeof trace) == XQ_OK);
    CHECK(strstr(trace, "prefill_token_custom") != NULL);
    CHECK(strstr(trace, "prefill_kv_build_custom") != NULL);
    CHECK(strstr(trace, "linear_attention_state_update_custom") != NULL);

    int32_t next = -1;
    CHECK(xq_decode_one(session, &next, &metrics) == XQ_OK);
    CHECK(next >= 0 && next < 8);
    CHECK(metrics.generated_tokens == 1);
    printf("decode_token %d\n", next);
    CHECK(print_hidden(session, "hidden_decode"));

    int32_t out[2] = {-1, -1};
    CHECK(xq_generate(session, prompt, 3, 2, out, 2, &metrics) == XQ_OK);
    CHECK(metrics.generated_tokens == 2);
    CHECK(metrics.decode_tokens_per_second >= 0.0);
    printf("generate_tokens %d %d\n", out[0], out[1]);
    CHECK(print_hidden(session, "hidden_generate"));

    CHECK(xq_get_kernel_trace_json(session, trace, sizeof trace) == XQ_OK);
    CHECK(strstr(trace, "attention_score_custom") != NULL);
    CHECK(strstr(trace, "attention_softmax_custom") != NULL);
    CHECK(strstr(trace, "attention_v_reduce_custom") != NULL);
    CHECK(strstr(trace, "lm_head_custom") != NULL);
    CHECK(strstr(trace, "sampling_greedy_custom") != NULL);
    CHECK(strstr(trace, "fallback_") == NULL);

    static char info[4096];
    CHECK(xq_get_backend_info(session, info, sizeof info) == XQ_OK);
    CHECK(strstr(info, "full_custom_decode=true") != NULL);
    CHECK(strstr(info, "fallback_ops=none") != NULL);

    xq_destroy(session);
    printf("ok\n");
    return 0;
}
