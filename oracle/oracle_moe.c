/*
 * CPU ORACLE — test infrastructure only (see oracle.h).  Mixture-of-experts
 * routing and combination as llama.cpp's MoE FFN computes them (ggml's
 * scalar ops; llama.cpp is not in the reference tree and its version is not
 * pinned): soft_max with the sum in double and p = e·(float)(1/sum), the
 * n_used largest p (equal p: the lower expert id), their weights optionally
 * divided by their double sum rounded to float, and the weighted sum of the
 * experts' outputs in choice order.  The MoE tensors are the ones Milda and
 * Sutra place with tensor buffer overrides (Milda/src/engine.cpp:860-885,
 * Sutra/src/llm_backends.cpp:1716-1747).
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>

void orc_moe_route(const float* logits, int n_expert, int n_used, int norm, int32_t* ids, float* weights) {
    float mx = -FLT_MAX;
    for (int i = 0; i < n_expert; ++i)
        if (logits[i] > mx) mx = logits[i];
    float* p = (float*)malloc(sizeof(float) * (size_t)n_expert);
    double sum = 0.0;
    for (int i = 0; i < n_expert; ++i) {
        p[i] = expf(logits[i] - mx);
        sum += (double)p[i];
    }
    const float scale = (float)(1.0 / sum);
    for (int i = 0; i < n_expert; ++i) p[i] *= scale;
    char* taken = (char*)calloc((size_t)n_expert, 1);
    double s = 0.0;
    for (int j = 0; j < n_used; ++j) {
        int best = -1;
        for (int i = 0; i < n_expert; ++i)
            if (!taken[i] && (best < 0 || p[i] > p[best])) best = i;
        taken[best] = 1;
        ids[j] = best;
        weights[j] = p[best];
        s += (double)p[best];
    }
    if (norm) {
        const float sf = (float)s;
        for (int j = 0; j < n_used; ++j) weights[j] = weights[j] / sf;
    }
    free(taken);
    free(p);
}

void orc_moe_combine(const float* y, const float* w, int n_used, int n, float* out) {
    for (int i = 0; i < n; ++i) {
        float acc = y[i] * w[0];
        for (int j = 1; j < n_used; ++j) acc = acc + y[(size_t)j * n + i] * w[j];
        out[i] = acc;
    }
}
