/*
 * localinfer -- the reference's single-machine CLI (src/bin/localinfer.c) on the B200 engine.
 *
 *   localinfer <model dir> [-t temperature] [-p topp] [-s seed] [-n steps] [-i prompt]
 *              [-z tokenizer] [-m generate|chat] [-y system prompt]
 *
 * Same flags, defaults and clamping (temperature 1.0, topp 0.9, steps 256 with 0 or more than
 * seq_len meaning seq_len, seed from the clock when 0, tokenizer python/tokenizer.bin), the same
 * generate loop (prompt tokens forced one position at a time, then sampled tokens; stop at token 1;
 * pieces printed as they come; "achieved tok/s" timed from the second position) and the same chat
 * loop.  The model runs on the current CUDA device (CUDA_VISIBLE_DEVICES picks it).
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "diolkos.h"
#include "safetensors.h"
#include "sampler.h"
#include "tensor.h"
#include "tokenizer.h"
#include "transformer.h"

static long time_in_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_REALTIME, &ts);
    return ts.tv_sec * 1000 + ts.tv_nsec / 1000000;
}

/* Parameter count of the loaded weights (embedding, norms, every matrix, classifier). */
static size_t count_params(const Transformer *t) {
    const Model *m = t->safetensors;
    size_t total = m->token_embedding_table->dim + m->rms_final_weight->dim + m->wcls->dim;
    for (int l = 0; l < t->config.n_layers; ++l) {
        const Layer *L = &m->layers[l];
        total += L->rms_att_weight->dim + L->rms_ffn_weight->dim + L->wq->dim + L->wk->dim + L->wv->dim + L->wo->dim +
                 L->w1->dim + L->w2->dim + L->w3->dim;
    }
    return total;
}

static float generate(Transformer *tf, Tokenizer *tok, Sampler *sampler, const char *prompt, int steps) {
    if (!prompt) prompt = "";
    int n_prompt = 0;
    int *prompt_tokens = malloc((strlen(prompt) + 3) * sizeof(int));
    encode(tok, prompt, 1, 0, prompt_tokens, &n_prompt);
    if (n_prompt < 1) {
        fprintf(stderr, "something is wrong, expected at least 1 prompt token\n");
        exit(EXIT_FAILURE);
    }
    long start = 0;
    int token = prompt_tokens[0], pos = 0, next = 0, pos_start = 0, stop = 0;
    /* The forced prompt positions (all but the last prompt token) run as one prefill on the GPU, which
     * leaves the KV cache as forward() at each of them would; their pieces print as the loop prints
     * them.  If the engine cannot prefill, the loop forwards them one by one. */
    const int pre = n_prompt - 1 < steps ? n_prompt - 1 : steps;
    if (pre > 0 && transformer_prefill(tf, prompt_tokens, pre) == 0) {
        while (pos < pre) {
            next = prompt_tokens[pos + 1];
            pos++;
            if (next == 1) {
                stop = 1;
                break;
            }
            safe_printf(decode(tok, token, next));
            token = next;
        }
        fflush(stdout);
    }
    while (!stop && pos < steps) {
        Tensor *logits = forward(tf, token, pos);
        next = pos < n_prompt - 1 ? prompt_tokens[pos + 1] : sample(sampler, data_f32(logits));
        pos++;
        if (next == 1) break;  /* BOS delimits sequences */
        safe_printf(decode(tok, token, next));
        fflush(stdout);
        token = next;
        if (start == 0) {
            start = time_in_ms();
            pos_start = pos;
        }
    }
    printf("\n");
    float tok_s = 0.0f;
    if (start && pos > pos_start) {  /* the positions forwarded after the first timed one */
        const long end = time_in_ms();
        tok_s = (float)(pos - pos_start) * 1000.0f / (float)(end > start ? end - start : 1);
        fprintf(stderr, "achieved tok/s: %.2f\n", tok_s);
    }
    free(prompt_tokens);
    return tok_s;
}

static void read_stdin(const char *guide, char *buf, size_t size) {
    printf("%s", guide);
    if (fgets(buf, (int)size, stdin)) {
        const size_t len = strlen(buf);
        if (len && buf[len - 1] == '\n') buf[len - 1] = '\0';
    } else {
        buf[0] = '\0';
    }
}

static void chat(Transformer *tf, Tokenizer *tok, Sampler *sampler, const char *cli_user, const char *cli_system,
                 int steps) {
    char system_prompt[512] = "", user_prompt[512] = "", rendered[1152];
    int *prompt_tokens = malloc(1152 * sizeof(int));
    int n_prompt = 0, user_idx = 0, next = 0, token, pos = 0;
    int user_turn = 1;
    while (pos < steps) {
        if (user_turn) {
            if (pos == 0) {
                if (cli_system) snprintf(system_prompt, sizeof system_prompt, "%s", cli_system);
                else read_stdin("Enter system prompt (optional): ", system_prompt, sizeof system_prompt);
            }
            if (pos == 0 && cli_user) snprintf(user_prompt, sizeof user_prompt, "%s", cli_user);
            else read_stdin("User: ", user_prompt, sizeof user_prompt);
            if (pos == 0 && system_prompt[0])
                snprintf(rendered, sizeof rendered, "[INST] <<SYS>>\n%s\n<</SYS>>\n\n%s [/INST]", system_prompt,
                         user_prompt);
            else
                snprintf(rendered, sizeof rendered, "<|im_start|>user\n%s<|im_end|>\n<|im_start|>assistant\n",
                         user_prompt);
            encode(tok, rendered, 1, 0, prompt_tokens, &n_prompt);
            user_idx = 0;
            user_turn = 0;
            printf("Assistant: ");
        }
        token = user_idx < n_prompt ? prompt_tokens[user_idx++] : next;
        if (token == 2) user_turn = 1;  /* EOS ends the assistant's turn */
        Tensor *logits = forward(tf, token, pos);
        next = sample(sampler, data_f32(logits));
        pos++;
        if (user_idx >= n_prompt && next != 2) {
            safe_printf(decode(tok, token, next));
            fflush(stdout);
        }
        if (next == 2) printf("\n");
    }
    printf("\nChat reached the max length of %d tokens.\n", steps);
    free(prompt_tokens);
}

static void error_usage(void) {
    fprintf(stderr,
            "Usage:   localinfer <model dir> [options]\n"
            "Example: localinfer models/llama2-7b -n 256 -i \"Once upon a time\"\n"
            "Options:\n"
            "  -t <float>  temperature in [0,inf], default 1.0\n"
            "  -p <float>  p value in top-p (nucleus) sampling in [0,1] default 0.9\n"
            "  -s <int>    random seed, default time(NULL)\n"
            "  -n <int>    number of steps to run for, default 256. 0 = max_seq_len\n"
            "  -i <string> input prompt\n"
            "  -z <string> optional path to custom tokenizer\n"
            "  -m <string> mode: generate|chat, default: generate\n"
            "  -y <string> (optional) system prompt in chat mode\n");
    exit(EXIT_FAILURE);
}

int main(int argc, char **argv) {
    const char *model_dir = NULL, *tokenizer_path = "python/tokenizer.bin", *mode = "generate";
    const char *prompt = NULL, *system_prompt = NULL;
    float temperature = 1.0f, topp = 0.9f;
    int steps = 256;
    unsigned long long seed = 0;
    const long t0 = time_in_ms();

    if (argc < 2) error_usage();
    model_dir = argv[1];
    for (int i = 2; i < argc; i += 2) {
        if (i + 1 >= argc || argv[i][0] != '-' || strlen(argv[i]) != 2) error_usage();
        const char *v = argv[i + 1];
        switch (argv[i][1]) {
            case 't': temperature = (float)atof(v); break;
            case 'p': topp = (float)atof(v); break;
            case 's': seed = (unsigned long long)atoi(v); break;
            case 'n': steps = atoi(v); break;
            case 'i': prompt = v; break;
            case 'z': tokenizer_path = v; break;
            case 'm': mode = v; break;
            case 'y': system_prompt = v; break;
            default: error_usage();
        }
    }
    if (seed == 0) seed = (unsigned int)time(NULL);
    if (temperature < 0.0f) temperature = 0.0f;
    if (topp < 0.0f || topp > 1.0f) topp = 0.9f;
    if (steps < 0) steps = 0;

    Transformer transformer;
    build_transformer_from_safetensors(&transformer, model_dir);
    if (steps == 0 || steps > transformer.config.seq_len) steps = transformer.config.seq_len;
    Tokenizer tokenizer;
    build_tokenizer(&tokenizer, tokenizer_path);
    Sampler sampler;
    build_sampler(&sampler, transformer.config.vocab_size, temperature, topp, seed);
    fprintf(stderr, "Initialization took %ld ms\n", time_in_ms() - t0);

    const size_t params = count_params(&transformer);
    fprintf(stderr, "Parameters: %zu (%.2f GB of weights read per token on the GPU)\n", params,
            (double)dk_model_weight_bytes(transformer_engine(&transformer)) / 1e9);

    if (strcmp(mode, "generate") == 0) {
        const float tok_s = generate(&transformer, &tokenizer, &sampler, prompt, steps);
        fprintf(stderr, "GMAC: %.1f\n", (double)tok_s * (double)params / 1e9);
    } else if (strcmp(mode, "chat") == 0) {
        chat(&transformer, &tokenizer, &sampler, prompt, system_prompt, steps);
    } else {
        fprintf(stderr, "unknown mode: %s\n", mode);
        error_usage();
    }
    free_sampler(&sampler);
    free_tokenizer(&tokenizer);
    free_transformer(&transformer);
    return 0;
}
