/*
 * client -- the reference's tensor-parallel CLI (src/bin/client.c) on the GPUs of one box.
 *
 *   client <model dir> [-t temperature] [-p topp] [-s seed] [-n steps] [-i prompt] [-z tokenizer]
 *          [-m generate] [-g gpus]
 *
 * The reference's client drives TCP workers that each hold a slice of every weight matrix
 * (src/bin/client.c, src/remote_workers.c).  Here the workers are GPUs of this box: the client forks
 * one process per GPU BEFORE any CUDA call; rank r builds its shard on GPU r
 * (build_transformer_tp), the ranks swap their exchange handles through a shared anonymous mapping,
 * and every rank runs the same forward() steps, the per-layer sums travelling over NVLink inside the
 * decode step.  Rank 0 encodes the prompt, samples (the other ranks' classifier rows reach it through
 * the mapping), prints, and tells the ranks the next token.
 *
 * Flags, defaults and the generate loop are the reference's (same as localinfer); -g <n> (this
 * build's) picks the number of GPUs, default 2 like the reference's two workers.  Chat mode is
 * served by localinfer.
 */
#include <sched.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/wait.h>
#include <time.h>
#include <unistd.h>

#include "diolkos.h"
#include "sampler.h"
#include "tensor.h"
#include "tokenizer.h"
#include "transformer.h"

#define MAX_RANKS 8

typedef struct {
    volatile int arrived;           /* sense-reversing barrier */
    volatile int generation;
    volatile int failed;            /* a rank gave up: everyone leaves */
    volatile int next;              /* the token rank 0 chose */
    unsigned char handles[MAX_RANKS][DK_COMM_HANDLE_BYTES];
    float logits[];                 /* vocab: every rank's classifier rows, gathered for rank 0 */
} Shared;

static long time_in_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_REALTIME, &ts);
    return ts.tv_sec * 1000 + ts.tv_nsec / 1000000;
}

/* Barrier over the ranks' processes; gives up (and marks the run failed) after 120 s, e.g. when a
 * rank died. */
static void barrier(Shared *sh, int world) {
    const int gen = sh->generation;
    if (__atomic_add_fetch(&sh->arrived, 1, __ATOMIC_ACQ_REL) == world) {
        __atomic_store_n(&sh->arrived, 0, __ATOMIC_RELAXED);
        __atomic_store_n(&sh->generation, gen + 1, __ATOMIC_RELEASE);
        return;
    }
    const long t0 = time_in_ms();
    while (__atomic_load_n(&sh->generation, __ATOMIC_ACQUIRE) == gen) {
        if (sh->failed || time_in_ms() - t0 > 120000) {
            sh->failed = 1;
            fprintf(stderr, "client: a rank stopped answering\n");
            exit(EXIT_FAILURE);
        }
        sched_yield();
    }
}

static void error_usage(void) {
    fprintf(stderr,
            "Usage:   client <model dir> [options]\n"
            "Example: client models/llama2-7b -n 256 -i \"Once upon a time\" -g 2\n"
            "Options:\n"
            "  -t <float>  temperature in [0,inf], default 1.0\n"
            "  -p <float>  p value in top-p (nucleus) sampling in [0,1] default 0.9\n"
            "  -s <int>    random seed, default time(NULL)\n"
            "  -n <int>    number of steps to run for, default 256. 0 = max_seq_len\n"
            "  -i <string> input prompt\n"
            "  -z <string> tokenizer path (default: python/tokenizer.bin)\n"
            "  -m <string> mode: generate (chat: use localinfer)\n"
            "  -g <int>    GPUs (tensor-parallel ranks, 1 to 8), default 2\n");
    exit(EXIT_FAILURE);
}

static int run_rank(int rank, int world, Shared *sh, const char *model_dir, const char *tokenizer_path,
                    const char *prompt, float temperature, float topp, unsigned long long seed, int steps) {
    /* rank 0 loads first, so that the Q8_0 cache files are written once; the others then map them */
    if (rank != 0) barrier(sh, world);
    Transformer t;
    memset(&t, 0, sizeof t);
    build_transformer_tp(&t, model_dir, rank, world, rank, sh->handles[rank]);
    if (rank == 0) barrier(sh, world);
    barrier(sh, world);  /* every handle is in the mapping */
    build_transformer_tp_connect(&t, sh->handles);
    if (steps == 0 || steps > t.config.seq_len) steps = t.config.seq_len;

    Tokenizer tok;
    build_tokenizer(&tok, tokenizer_path);
    Sampler sampler;
    build_sampler(&sampler, t.config.vocab_size, temperature, topp, seed);
    if (!prompt) prompt = "";
    int n_prompt = 0;
    int *prompt_tokens = malloc((strlen(prompt) + 3) * sizeof(int));
    encode(&tok, prompt, 1, 0, prompt_tokens, &n_prompt);  /* the same tokens on every rank */
    if (n_prompt < 1) {
        fprintf(stderr, "something is wrong, expected at least 1 prompt token\n");
        exit(EXIT_FAILURE);
    }
    int row0, row1;
    transformer_logit_rows(&t, &row0, &row1);
    barrier(sh, world);

    long start = 0;
    int token = prompt_tokens[0], pos = 0, next = 0, pos_start = 0, stop = 0;
    /* the forced prompt positions as one prefill on every rank (pieces printed as the loop prints them) */
    const int pre = n_prompt - 1 < steps ? n_prompt - 1 : steps;
    if (pre > 0 && transformer_prefill(&t, prompt_tokens, pre) == 0) {
        while (pos < pre) {
            next = prompt_tokens[pos + 1];
            pos++;
            if (next == 1) {
                stop = 1;
                break;
            }
            if (rank == 0) safe_printf(decode(&tok, token, next));
            token = next;
        }
        if (rank == 0) fflush(stdout);
    }
    while (!stop && pos < steps) {
        Tensor *logits = forward(&t, token, pos);
        if (pos < n_prompt - 1) {
            next = prompt_tokens[pos + 1];
        } else {
            float *lg = data_f32(logits);
            if (rank != 0) memcpy(sh->logits + row0, lg + row0, (size_t)(row1 - row0) * sizeof(float));
            barrier(sh, world);
            if (rank == 0) {
                for (int r = 1; r < world; ++r) {
                    const int per = (t.config.vocab_size + world - 1) / world;
                    const int b = r * per, e = b + per < t.config.vocab_size ? b + per : t.config.vocab_size;
                    memcpy(lg + b, sh->logits + b, (size_t)(e - b) * sizeof(float));
                }
                sh->next = sample(&sampler, lg);
            }
            barrier(sh, world);
            next = sh->next;
        }
        pos++;
        if (next == 1) break;
        if (rank == 0) {
            safe_printf(decode(&tok, token, next));
            fflush(stdout);
        }
        token = next;
        if (start == 0) {
            start = time_in_ms();
            pos_start = pos;
        }
    }
    if (rank == 0) {
        printf("\n");
        if (start && pos > pos_start) {
            const long end = time_in_ms();
            fprintf(stderr, "achieved tok/s: %.2f (%d GPUs)\n",
                    (double)(pos - pos_start) * 1000.0 / (double)(end > start ? end - start : 1), world);
        }
    }
    barrier(sh, world);  /* nobody leaves the exchange while another rank still steps */
    free(prompt_tokens);
    free_sampler(&sampler);
    free_tokenizer(&tok);
    free_transformer(&t);
    return 0;
}

int main(int argc, char **argv) {
    const char *model_dir, *tokenizer_path = "python/tokenizer.bin", *mode = "generate";
    const char *prompt = NULL;
    float temperature = 1.0f, topp = 0.9f;
    int steps = 256, world = 2;
    unsigned long long seed = 0;
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
            case 'y': break;  /* chat system prompt: chat mode is localinfer's */
            case 'g': world = atoi(v); break;
            default: error_usage();
        }
    }
    if (strcmp(mode, "generate") != 0) {
        fprintf(stderr, "client: mode %s is not served here (chat: use localinfer)\n", mode);
        error_usage();
    }
    if (world < 1 || world > MAX_RANKS) error_usage();
    if (seed == 0) seed = (unsigned int)time(NULL);
    if (temperature < 0.0f) temperature = 0.0f;
    if (topp < 0.0f || topp > 1.0f) topp = 0.9f;
    if (steps < 0) steps = 0;

    /* the mapping is sized for vocabularies up to 1M entries (4 MB) */
    const size_t bytes = sizeof(Shared) + (size_t)(1 << 20) * sizeof(float);
    Shared *sh = mmap(NULL, bytes, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_ANONYMOUS, -1, 0);
    if (sh == MAP_FAILED) {
        perror("mmap");
        return EXIT_FAILURE;
    }
    memset(sh, 0, sizeof(Shared));
    fflush(stdout);
    pid_t pids[MAX_RANKS] = {0};
    for (int r = 1; r < world; ++r) {
        const pid_t p = fork();  /* before any CUDA call: each rank initialises its own context */
        if (p < 0) {
            perror("fork");
            sh->failed = 1;
            return EXIT_FAILURE;
        }
        if (p == 0) {
            const int rc = run_rank(r, world, sh, model_dir, tokenizer_path, prompt, temperature, topp, seed, steps);
            fflush(stdout);
            _exit(rc);
        }
        pids[r] = p;
    }
    int rc = run_rank(0, world, sh, model_dir, tokenizer_path, prompt, temperature, topp, seed, steps);
    for (int r = 1; r < world; ++r) {
        int status = 0;
        if (waitpid(pids[r], &status, 0) < 0 || !WIFEXITED(status) || WEXITSTATUS(status) != 0) rc = EXIT_FAILURE;
    }
    munmap(sh, bytes);
    return rc;
}
