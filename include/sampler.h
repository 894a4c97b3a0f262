/*
 * sampler.h -- the reference's token sampler (src/sampler.h), computed on the GPU.
 *
 * sample() takes HOST logits, like the reference: temperature 0 is greedy argmax (first index wins
 * ties); otherwise softmax(logits / temperature) and either plain multinomial sampling (topp <= 0
 * or >= 1) or top-p (nucleus) sampling, with the reference's xorshift random stream on the host
 * giving the coin (so a seed reproduces the same coin sequence as the reference).  The arithmetic
 * runs in dk_sample (diolkos.h), on device buffers the library keeps per device (not re-entrant,
 * like the reference's sampler and utils).
 */
#ifndef DIOLKOS_SAMPLER_H
#define DIOLKOS_SAMPLER_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    float prob;
    int index;
} ProbIndex;

/* Same layout as the reference's (callers allocate it).  probindex is allocated like the
 * reference's but unused: the GPU needs no sort buffer. */
typedef struct {
    int vocab_size;
    ProbIndex *probindex;
    float temperature;
    float topp;
    unsigned long long rng_state;
} Sampler;

void build_sampler(Sampler *sampler, int vocab_size, float temperature, float topp, unsigned long long rng_seed);
void free_sampler(Sampler *sampler);
/* The next token from host logits[vocab_size] (the logits are not modified). */
int sample(Sampler *sampler, float *logits);
/* The reference's xorshift* stream (src/sampler.c:96-106). */
unsigned int random_u32(unsigned long long *state);
float random_f32(unsigned long long *state);

#ifdef __cplusplus
}
#endif
#endif
