/*
 * tokenizer.h -- the reference's BPE tokenizer (src/tokenizer.h) over a llama2.c-format
 * tokenizer.bin (vocab size, max token length, bos, eos as int32, then per token: fp32 score, int32
 * length, bytes).  Host string processing.
 */
#ifndef DIOLKOS_TOKENIZER_H
#define DIOLKOS_TOKENIZER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    const char *str;
    int id;
} TokenIndex;

typedef struct {
    char **vocab;
    float *vocab_scores;
    TokenIndex *sorted_vocab;
    int vocab_size;
    unsigned int max_token_length;
    unsigned char byte_pieces[512]; /* the 256 single-byte strings */
    int bos_id;
    int eos_id;
} Tokenizer;

void build_tokenizer(Tokenizer *t, const char *tokenizer_path);
void free_tokenizer(Tokenizer *t);
/* The text of `token` following `prev_token` (a leading space is dropped after BOS; <0xNN> byte
 * tokens become the raw byte). */
char *decode(Tokenizer *t, int prev_token, int token);
/* Print a piece unless it is a single non-printable byte. */
void safe_printf(const char *piece);
/* BPE-encode `text` into tokens (bos / eos != 0 add token 1 / 2); tokens needs strlen(text) + 3 slots. */
void encode(Tokenizer *t, const char *text, int8_t bos, int8_t eos, int *tokens, int *n_tokens);
/* Index of `str` in the sorted vocabulary, or -1. */
int str_lookup(const char *str, TokenIndex *sorted_vocab, int vocab_size);

#ifdef __cplusplus
}
#endif
#endif
