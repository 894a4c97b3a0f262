/*
 * sampler.c -- the reference's sampler API (src/sampler.c) with the arithmetic on the GPU.
 *
 * The random stream stays on the host and is consumed exactly like the reference's: one
 * random_f32 draw per sample() call with temperature > 0, none at temperature 0
 * (src/sampler.c:108-131).  The logits are copied to the device, dk_sample picks the token and, at
 * temperature > 0, the probabilities come back into the caller's logits buffer, which the
 * reference also overwrites with them.
 */
#include <stdio.h>
#include <stdlib.h>

#include <cuda_runtime_api.h>

#include "diolkos.h"
#include "host_internal.h"
#include "sampler.h"

void build_sampler(Sampler *s, int vocab_size, float temperature, float topp, unsigned long long rng_seed) {
    s->vocab_size = vocab_size;
    s->temperature = temperature;
    s->topp = topp;
    s->rng_state = rng_seed;
    /* allocated like the reference's sort buffer; the GPU sampler does not use it */
    s->probindex = host_malloc((size_t)(vocab_size > 0 ? vocab_size : 1) * sizeof(ProbIndex));
}

void free_sampler(Sampler *s) {
    free(s->probindex);
    s->probindex = NULL;
}

/* Device logits + token, grown to the largest vocabulary seen (the Sampler keeps the reference's
 * layout, so the buffer lives here; one per process like the reference's own scratch). */
static dev_buf g_sample;

unsigned int random_u32(unsigned long long *state) {
    /* xorshift* (Marsaglia's xorshift with a multiplicative output step), 64-bit state */
    unsigned long long x = *state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    return (unsigned int)((x * 0x2545F4914F6CDD1Dull) >> 32);
}

float random_f32(unsigned long long *state) { return (float)(random_u32(state) >> 8) / 16777216.0f; }

int sample(Sampler *s, float *logits) {
    const int n = s->vocab_size;
    const size_t bytes = (size_t)n * sizeof(float);
    char *base = dev_reserve(&g_sample, (bytes + 15) / 16 * 16 + 16);
    float *d_logits = (float *)base;
    int *d_out = (int *)(base + (bytes + 15) / 16 * 16);
    host_check_cuda(cudaMemcpy(d_logits, logits, bytes, cudaMemcpyHostToDevice), "sample: copy logits");
    int next = 0;
    if (s->temperature == 0.0f) {
        host_check(dk_sample(d_logits, n, 0.0f, s->topp, 0.0f, NULL, d_out, NULL), "sample");
    } else {
        const float coin = random_f32(&s->rng_state);
        host_check(dk_sample(d_logits, n, s->temperature, s->topp, coin, d_logits, d_out, NULL), "sample");
        host_check_cuda(cudaMemcpy(logits, d_logits, bytes, cudaMemcpyDeviceToHost), "sample: copy probabilities");
    }
    host_check_cuda(cudaMemcpy(&next, d_out, sizeof next, cudaMemcpyDeviceToHost), "sample: copy token");
    return next;
}
