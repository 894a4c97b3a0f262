/*
 * sampler.h -- the reference's token sampler (src/sampler.h), computed on the GPU.
 *
 * sample() takes HOST logits, like the reference: temperature 0 is greedy argmax (first index wins
 * ties); otherwise softmax(logits / temperature) and either plain multinomial sampling (topp <= 0
 * or >= 1) or top-p (nucleus) sampling, with the reference's xorshift random stream on the host
 * giving the coin (so a seed reproduces the same coin sequence as the reference).  The arithmetic
 * runs in dk_sample (diolkos.h).
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

typedef struct {
    int vocab_size;
    ProbIndex *probindex;  /* unused here (the GPU needs no sort buffer); kept for compatibility */
    float temperature;
    float topp;
    unsigned long long rng_state;
    void *device_buf;      /* logits and result on the device */
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
