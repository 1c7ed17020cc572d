/*
 * CPU ORACLE — test infrastructure only (see oracle.h).  The sampler chain.
 *
 * Milda builds its chain in rebuild_sampler (Milda/src/engine.cpp:1321-1384):
 * penalties (last 64 tokens, its repeat penalty, no frequency or presence
 * penalty), then greedy when the temperature is <= 0, else top_k, top_p(p, 1),
 * min_p(p, 1), temp and dist(seed).  It samples with llama_sampler_sample
 * (:1970) and accepts the token again (:2029).  The samplers are llama.cpp's
 * (not in the reference tree, version not pinned) and are restated here from
 * their published source; dist draws with std::discrete_distribution and
 * std::mt19937 as the GNU C++ library implements them (pinned against the
 * library by tests/golden/make_sampler_golden.py).  Equal logits sort by
 * lower token id.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

enum { MT_N = 624, RING_MAX = 4096 };

struct orc_sampler {
    int last_n;
    float rep, freq, pres;
    int top_k;
    float top_p, min_p, temp;
    uint32_t seed;
    int ring_len, ring_head;
    int32_t ring[RING_MAX];
    uint32_t mt[MT_N];
    int mti;
};

/* ---- std::mt19937 (Matsumoto & Nishimura 1998; C++ [rand.eng.mers]) ---- */
static void mt_seed(orc_sampler* s, uint32_t seed) {
    s->mt[0] = seed;
    for (int k = 1; k < MT_N; ++k) s->mt[k] = 1812433253u * (s->mt[k - 1] ^ (s->mt[k - 1] >> 30)) + (uint32_t)k;
    s->mti = MT_N;
}

static uint32_t mt_next(orc_sampler* s) {
    if (s->mti >= MT_N) {
        for (int k = 0; k < MT_N; ++k) {
            const uint32_t y = (s->mt[k] & 0x80000000u) | (s->mt[(k + 1) % MT_N] & 0x7FFFFFFFu);
            s->mt[k] = s->mt[(k + 397) % MT_N] ^ (y >> 1) ^ ((y & 1u) ? 0x9908B0DFu : 0u);
        }
        s->mti = 0;
    }
    uint32_t y = s->mt[s->mti++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9D2C5680u;
    y ^= (y << 15) & 0xEFC60000u;
    y ^= y >> 18;
    return y;
}

void orc_mt19937(uint32_t seed, uint32_t* out, int n) {
    orc_sampler s;
    mt_seed(&s, seed);
    for (int i = 0; i < n; ++i) out[i] = mt_next(&s);
}

/* std::generate_canonical<double, 53> over a 32-bit engine (GNU C++
 * library): two draws, (r1 + r2·2^32)/2^64, kept below 1. */
static double canonical(orc_sampler* s) {
    const double r1 = (double)mt_next(s);
    const double r2 = (double)mt_next(s);
    double u = (r1 + r2 * 4294967296.0) / 18446744073709551616.0;
    if (u >= 1.0) u = nextafter(1.0, 0.0);
    return u;
}

/* std::discrete_distribution<int>(p, p + n)(rng) (GNU C++ library): the
 * weights summed in double, each divided by the sum, running sums with the
 * last set to 1, and the first running sum not below u among the first n-1;
 * fewer than two weights: 0 without a draw. */
int orc_discrete_draw(orc_sampler* s, const float* p, int n) {
    if (n < 2) return 0;
    double sum = 0.0;
    for (int i = 0; i < n; ++i) sum += (double)p[i];
    double* cp = (double*)malloc(sizeof(double) * (size_t)n);
    double run = 0.0;
    for (int i = 0; i < n; ++i) {
        run += (double)p[i] / sum;
        cp[i] = run;
    }
    cp[n - 1] = 1.0;
    const double u = canonical(s);
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi) / 2;
        if (cp[mid] < u) lo = mid + 1;
        else hi = mid;
    }
    free(cp);
    return lo;
}

orc_sampler* orc_sampler_new(int last_n, float rep, float freq, float pres, int top_k, float top_p, float min_p,
                             float temp, uint32_t seed) {
    if (last_n < 0 || last_n > RING_MAX) return NULL;
    orc_sampler* s = (orc_sampler*)calloc(1, sizeof(orc_sampler));
    s->last_n = last_n;
    s->rep = rep;
    s->freq = freq;
    s->pres = pres;
    s->top_k = top_k;
    s->top_p = top_p;
    s->min_p = min_p;
    s->temp = temp;
    s->seed = seed;
    orc_sampler_reset(s);
    return s;
}

void orc_sampler_free(orc_sampler* s) { free(s); }

/* llama_sampler_reset: the penalties forget their window, dist re-seeds. */
void orc_sampler_reset(orc_sampler* s) {
    s->ring_len = 0;
    s->ring_head = 0;
    mt_seed(s, s->seed);
}

/* llama_sampler_accept: the penalties' ring of the last last_n tokens. */
void orc_sampler_accept(orc_sampler* s, int32_t tok) {
    if (s->last_n <= 0) return;
    if (s->ring_len < s->last_n) {
        s->ring[(s->ring_head + s->ring_len) % s->last_n] = tok;
        ++s->ring_len;
    } else {
        s->ring[s->ring_head] = tok;
        s->ring_head = (s->ring_head + 1) % s->last_n;
    }
}

typedef struct {
    int32_t id;
    float logit, p;
} cand;

static int cand_desc(const void* a, const void* b) {
    const cand* x = (const cand*)a;
    const cand* y = (const cand*)b;
    if (x->logit != y->logit) return x->logit > y->logit ? -1 : 1;
    return x->id < y->id ? -1 : (x->id > y->id);
}

/* llama_sampler_softmax_impl on sorted candidates. */
static void softmax_sorted(cand* c, int n) {
    const float mx = c[0].logit;
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        c[i].p = expf(c[i].logit - mx);
        sum += c[i].p;
    }
    for (int i = 0; i < n; ++i) c[i].p /= sum;
}

int32_t orc_sampler_sample(orc_sampler* s, const float* logits, int n_vocab) {
    cand* c = (cand*)malloc(sizeof(cand) * (size_t)n_vocab);
    for (int v = 0; v < n_vocab; ++v) {
        c[v].id = v;
        c[v].logit = logits[v];
        c[v].p = 0.0f;
    }
    /* penalties */
    if (s->last_n != 0 && !(s->rep == 1.0f && s->freq == 0.0f && s->pres == 0.0f)) {
        int* count = (int*)calloc((size_t)n_vocab, sizeof(int));
        for (int e = 0; e < s->ring_len; ++e) {
            const int t = s->ring[(s->ring_head + e) % s->last_n];
            if (t >= 0 && t < n_vocab) ++count[t];
        }
        for (int v = 0; v < n_vocab; ++v) {
            if (count[v] == 0) continue;
            float x = c[v].logit;
            x = x <= 0.0f ? x * s->rep : x / s->rep;
            x -= (float)count[v] * s->freq + (float)(count[v] > 0) * s->pres;
            c[v].logit = x;
        }
        free(count);
    }
    int pick = 0, size = n_vocab;
    if (s->temp <= 0.0f) {
        for (int v = 1; v < n_vocab; ++v)
            if (c[v].logit > c[pick].logit) pick = v;
    } else {
        qsort(c, (size_t)n_vocab, sizeof(cand), cand_desc);
        if (s->top_k > 0 && s->top_k < size) size = s->top_k;
        if (s->top_p > 0.0f && s->top_p < 1.0f) {
            softmax_sorted(c, size);
            float run = 0.0f;
            int last = size;
            for (int i = 0; i < size; ++i) {
                run += c[i].p;
                if (run >= s->top_p && i + 1 >= 1) {
                    last = i + 1;
                    break;
                }
            }
            size = last;
        }
        if (s->min_p > 0.0f) {
            const float min_logit = c[0].logit + logf(s->min_p);
            int i = 1;
            for (; i < size; ++i)
                if (c[i].logit < min_logit) break;
            size = i;
        }
        for (int i = 0; i < size; ++i) c[i].logit /= s->temp;
        softmax_sorted(c, size);
        float* p = (float*)malloc(sizeof(float) * (size_t)size);
        for (int i = 0; i < size; ++i) p[i] = c[i].p;
        pick = orc_discrete_draw(s, p, size);
        free(p);
    }
    const int32_t tok = c[pick].id;
    free(c);
    orc_sampler_accept(s, tok);
    return tok;
}
