/*
 * tokenizer.c -- the reference's BPE tokenizer (src/tokenizer.c) on a llama2.c tokenizer.bin.
 *
 * encode follows the reference's rules (src/tokenizer.c:93-209): optional BOS (id 1); a dummy " "
 * piece when the text is not empty; the text split into UTF-8 code points (a leading byte plus at
 * most three continuation bytes), each looked up as a piece, or byte-fallback ids (byte + 3) when it
 * is not in the vocabulary; then repeatedly the adjacent pair whose concatenation is the
 * highest-scoring piece is merged, the leftmost pair winning ties; optional EOS (id 2).
 *
 * The merge loop here keeps the tokens in a linked list and the candidate pairs in a max-heap
 * ordered by (score, leftmost position), so a prompt of n pieces costs O(n log n) lookups instead of
 * a rescan of every pair after each merge; the sequence of merges, and so the result, is the same.
 */
#include <ctype.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "host_internal.h"
#include "tokenizer.h"

static int cmp_token_index(const void *a, const void *b) {
    return strcmp(((const TokenIndex *)a)->str, ((const TokenIndex *)b)->str);
}

__attribute__((noreturn)) static void tok_fail(const char *what, const char *path, int i) {
    fprintf(stderr, "tokenizer %s: %s (entry %d)\n", path, what, i);
    exit(EXIT_FAILURE);
}

void build_tokenizer(Tokenizer *t, const char *tokenizer_path) {
    FILE *f = fopen(tokenizer_path, "rb");
    if (!f) {
        fprintf(stderr, "couldn't load %s\n", tokenizer_path);
        exit(EXIT_FAILURE);
    }
    int hdr[4];
    if (fread(hdr, sizeof(int), 4, f) != 4) tok_fail("short header", tokenizer_path, -1);
    if (hdr[0] <= 0 || hdr[1] < 0) tok_fail("bad header", tokenizer_path, -1);
    t->vocab_size = hdr[0];
    t->max_token_length = (unsigned)hdr[1];
    t->bos_id = hdr[2];
    t->eos_id = hdr[3];
    t->vocab = host_malloc((size_t)t->vocab_size * sizeof(char *));
    t->vocab_scores = host_malloc((size_t)t->vocab_size * sizeof(float));
    t->sorted_vocab = NULL;
    for (int b = 0; b < 256; ++b) {
        t->byte_pieces[2 * b] = (unsigned char)b;
        t->byte_pieces[2 * b + 1] = 0;
    }
    for (int i = 0; i < t->vocab_size; ++i) {
        int len = 0;
        if (fread(&t->vocab_scores[i], sizeof(float), 1, f) != 1) tok_fail("short score", tokenizer_path, i);
        if (fread(&len, sizeof(int), 1, f) != 1 || len < 0) tok_fail("bad piece length", tokenizer_path, i);
        t->vocab[i] = host_malloc((size_t)len + 1);
        if (len && fread(t->vocab[i], 1, (size_t)len, f) != (size_t)len) tok_fail("short piece", tokenizer_path, i);
        t->vocab[i][len] = '\0';
    }
    fclose(f);
}

void free_tokenizer(Tokenizer *t) {
    for (int i = 0; i < t->vocab_size; ++i) free(t->vocab[i]);
    free(t->vocab);
    free(t->vocab_scores);
    free(t->sorted_vocab);
    t->vocab = NULL;
    t->vocab_scores = NULL;
    t->sorted_vocab = NULL;
}

char *decode(Tokenizer *t, int prev_token, int token) {
    char *piece = t->vocab[token];
    /* after BOS (id 1) the sentencepiece decoder drops one leading space */
    if (prev_token == 1 && piece[0] == ' ') piece++;
    /* raw-byte pieces are spelled <0xNN> */
    unsigned char byte_val;
    if (sscanf(piece, "<0x%02hhX>", &byte_val) == 1) piece = (char *)t->byte_pieces + 2 * byte_val;
    return piece;
}

void safe_printf(const char *piece) {
    if (!piece || !piece[0]) return;
    if (!piece[1]) {
        const unsigned char b = (unsigned char)piece[0];
        if (!(isprint(b) || isspace(b))) return;  /* a lone control byte */
    }
    printf("%s", piece);
}

int str_lookup(const char *str, TokenIndex *sorted_vocab, int vocab_size) {
    const TokenIndex key = {str, 0};
    const TokenIndex *hit = bsearch(&key, sorted_vocab, (size_t)vocab_size, sizeof(TokenIndex), cmp_token_index);
    return hit ? hit->id : -1;
}

/* ---- merge heap ------------------------------------------------------------------------------ */
typedef struct {
    float score;
    int left, right;         /* node indices of the pair */
    unsigned vl, vr;         /* their versions when the pair was scored */
    int id;                  /* the merged piece */
} merge_cand;

typedef struct {
    merge_cand *a;
    size_t n, cap;
} merge_heap;

/* Higher score first; on equal scores the leftmost pair (node indices follow text order). */
static int cand_before(const merge_cand *x, const merge_cand *y) {
    if (x->score != y->score) return x->score > y->score;
    return x->left < y->left;
}

static void heap_push(merge_heap *h, merge_cand c) {
    if (h->n == h->cap) {
        h->cap = h->cap ? 2 * h->cap : 64;
        merge_cand *na = realloc(h->a, h->cap * sizeof(merge_cand));
        if (!na) {
            fprintf(stderr, "encode: out of memory\n");
            exit(EXIT_FAILURE);
        }
        h->a = na;
    }
    size_t i = h->n++;
    while (i > 0) {
        const size_t p = (i - 1) / 2;
        if (!cand_before(&c, &h->a[p])) break;
        h->a[i] = h->a[p];
        i = p;
    }
    h->a[i] = c;
}

static merge_cand heap_pop(merge_heap *h) {
    const merge_cand top = h->a[0];
    const merge_cand last = h->a[--h->n];
    size_t i = 0;
    for (;;) {
        size_t c = 2 * i + 1;
        if (c >= h->n) break;
        if (c + 1 < h->n && cand_before(&h->a[c + 1], &h->a[c])) c++;
        if (!cand_before(&h->a[c], &last)) break;
        h->a[i] = h->a[c];
        i = c;
    }
    if (h->n) h->a[i] = last;
    return top;
}

typedef struct {
    Tokenizer *t;
    int *tok, *next, *prev;
    unsigned *ver;
    char *buf;
    size_t buf_len;
    merge_heap heap;
} merger;

/* Score the pair (l, r) and queue it when its concatenation is a piece the reference would take
 * (score above its -1e10 floor). */
static void consider(merger *m, int l, int r) {
    if (l < 0 || r < 0) return;
    const char *a = m->t->vocab[m->tok[l]], *b = m->t->vocab[m->tok[r]];
    const size_t la = strlen(a), lb = strlen(b);
    if (la + lb + 1 > m->buf_len) {
        m->buf_len = 2 * (la + lb + 1);
        free(m->buf);
        m->buf = host_malloc(m->buf_len);
    }
    memcpy(m->buf, a, la);
    memcpy(m->buf + la, b, lb + 1);
    const int id = str_lookup(m->buf, m->t->sorted_vocab, m->t->vocab_size);
    if (id < 0) return;
    const float score = m->t->vocab_scores[id];
    if (!(score > -1e10f)) return;
    const merge_cand c = {score, l, r, m->ver[l], m->ver[r], id};
    heap_push(&m->heap, c);
}

void encode(Tokenizer *t, const char *text, int8_t bos, int8_t eos, int *tokens, int *n_tokens) {
    if (!text) {
        fprintf(stderr, "cannot encode NULL text\n");
        exit(EXIT_FAILURE);
    }
    if (!t->sorted_vocab) {
        t->sorted_vocab = host_malloc((size_t)t->vocab_size * sizeof(TokenIndex));
        for (int i = 0; i < t->vocab_size; ++i) {
            t->sorted_vocab[i].str = t->vocab[i];
            t->sorted_vocab[i].id = i;
        }
        qsort(t->sorted_vocab, (size_t)t->vocab_size, sizeof(TokenIndex), cmp_token_index);
    }

    int n = 0;
    if (bos) tokens[n++] = 1;
    if (text[0]) {
        const int space = str_lookup(" ", t->sorted_vocab, t->vocab_size);
        if (space < 0) {
            fprintf(stderr, "encode: the vocabulary has no \" \" piece\n");
            exit(EXIT_FAILURE);
        }
        tokens[n++] = space;
    }
    /* code points: a byte plus the continuation bytes (10xxxxxx) after it, four bytes at most */
    char cp[5];
    for (const unsigned char *c = (const unsigned char *)text; *c;) {
        size_t len = 0;
        cp[len++] = (char)*c++;
        while (len < 4 && (*c & 0xC0) == 0x80) cp[len++] = (char)*c++;
        cp[len] = '\0';
        const int id = str_lookup(cp, t->sorted_vocab, t->vocab_size);
        if (id >= 0) {
            tokens[n++] = id;
        } else {
            for (size_t i = 0; i < len; ++i) tokens[n++] = (unsigned char)cp[i] + 3;
        }
    }

    if (n > 1) {
        merger m = {0};
        m.t = t;
        m.tok = tokens;
        m.next = host_malloc((size_t)n * sizeof(int));
        m.prev = host_malloc((size_t)n * sizeof(int));
        m.ver = host_calloc((size_t)n, sizeof(unsigned));
        for (int i = 0; i < n; ++i) {
            m.next[i] = i + 1 < n ? i + 1 : -1;
            m.prev[i] = i - 1;
        }
        for (int i = 0; i + 1 < n; ++i) consider(&m, i, i + 1);
        while (m.heap.n) {
            const merge_cand c = heap_pop(&m.heap);
            if (m.ver[c.left] != c.vl || m.ver[c.right] != c.vr || m.next[c.left] != c.right) continue;  /* stale */
            /* merge right into left */
            tokens[c.left] = c.id;
            m.ver[c.left]++;
            m.ver[c.right]++;
            const int after = m.next[c.right];
            m.next[c.left] = after;
            if (after >= 0) m.prev[after] = c.left;
            m.next[c.right] = -1;
            consider(&m, m.prev[c.left], c.left);
            consider(&m, c.left, after);
        }
        /* compact the surviving nodes in order */
        int k = 0;
        for (int i = 0; i >= 0; i = m.next[i]) tokens[k++] = tokens[i];
        n = k;
        free(m.next);
        free(m.prev);
        free(m.ver);
        free(m.buf);
        free(m.heap.a);
    }
    if (eos) tokens[n++] = 2;
    *n_tokens = n;
}
