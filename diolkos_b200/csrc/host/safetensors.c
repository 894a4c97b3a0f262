/*
 * safetensors.c -- load_safetensors (reference src/safetensors.c:17-405): a HF LLaMA-2 directory
 * to host tensors, with the reference's Q8_0 cache.
 *
 *  * config.json: hidden_size, num_hidden_layers, num_attention_heads, num_key_value_heads,
 *    vocab_size, intermediate_size, max_position_embeddings (src/safetensors.c:290-300).
 *  * every "*.safetensors" file of the directory (in name order): 8-byte little-endian header
 *    length, JSON header, tensor data (src/safetensors.c:150-166).  A tensor name is taken from the
 *    first file that has it.
 *  * names and targets (src/safetensors.c:171-263): model.embed_tokens.weight and lm_head.weight
 *    Q8_0 [vocab x dim]; model.norm.weight F32 [dim]; model.layers.L.{input_layernorm,
 *    post_attention_layernorm}.weight F32 [dim]; model.layers.L.self_attn.{q,k,v,o}_proj.weight and
 *    model.layers.L.mlp.{gate,down,up}_proj.weight Q8_0.  A size mismatch or a missing tensor exits
 *    with a message.
 *  * cache (src/safetensors.c:57-114): ./cache/<directory basename>/<name>-<Q8_0|F32>.tensor holds
 *    the converted tensor (int8 values then fp32 scales for Q8_0).  When it exists it is mapped and
 *    used as is; otherwise the tensor is converted -- quantised on the GPU, bit-identical to the
 *    reference's convert_bf16_q8_0 / convert_f16_q8_0 / convert_f32_q8 -- and the file is written.
 *    Unlike the reference, ./cache itself is created when missing.
 */
#include <dirent.h>
#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "host_internal.h"
#include "safetensors.h"
#include "tensor.h"
#include "utils.h"

__attribute__((noreturn)) static void die(const char *fmt, const char *a, const char *b) {
    fprintf(stderr, fmt, a, b);
    fputc('\n', stderr);
    exit(EXIT_FAILURE);
}

/* A file mapped read-only; NULL when it cannot be opened or mapped (size in *size). */
static void *map_file(const char *path, size_t *size) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return NULL;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        close(fd);
        return NULL;
    }
    void *p = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return NULL;
    *size = (size_t)st.st_size;
    return p;
}

static void make_dir(const char *path) {
    if (mkdir(path, 0755) != 0 && errno != EEXIST) die("Failed to create cache directory %s%s", path, "");
}

/* The tensor `name` (header entry `entry`) as `target`, from the cache or converted. */
static Tensor *load_tensor(const js_node *entry, const char *model_name, const uint8_t *data, size_t data_bytes,
                           const char *name, size_t expected, quant_t target) {
    const js_node *dtype = js_get(entry, "dtype");
    quant_t src_type;
    size_t item;
    if (dtype && dtype->kind == JS_STR && strcmp(dtype->str, "F32") == 0) { src_type = F32; item = 4; }
    else if (dtype && dtype->kind == JS_STR && strcmp(dtype->str, "BF16") == 0) { src_type = BF16; item = 2; }
    else if (dtype && dtype->kind == JS_STR && strcmp(dtype->str, "F16") == 0) { src_type = F16; item = 2; }
    else die("Unsupported dtype for %s: %s", name, dtype && dtype->kind == JS_STR ? dtype->str : "(none)");

    const js_node *shape = js_get(entry, "shape");
    if (!shape || shape->kind != JS_ARR) die("Failed to get tensor shape for %s%s", name, "");
    size_t vdim = 1, hdim = 1;
    for (int i = 0; i < shape->n && i < 2; ++i) {
        if (shape->kids[i].kind != JS_NUM || shape->kids[i].num < 0) die("Bad shape for %s%s", name, "");
        if (i == 0) vdim = (size_t)shape->kids[i].num;
        else hdim = (size_t)shape->kids[i].num;
    }
    const size_t dim = vdim * hdim;
    if (dim != expected) {
        fprintf(stderr, "Tensor size mismatch for %s: expected %zu, got %zu\n", name, expected, dim);
        exit(EXIT_FAILURE);
    }

    char cache_name[1024];
    snprintf(cache_name, sizeof cache_name, "cache/%s/%s-%s.tensor", model_name, name, quant_t_to_string(target));
    size_t cache_bytes = 0;
    void *cached = map_file(cache_name, &cache_bytes);
    if (cached) {
        Tensor *t = host_calloc(1, sizeof(Tensor));
        t->type = target;
        t->dim = dim;
        t->vdim = vdim;
        t->hdim = hdim;
        if (cache_bytes < Tensor_storage_size(t)) die("Cache file %s is truncated%s", cache_name, "");
        t->data = (TensorData *)cached;
        if (target == Q8_0) t->scale = (float *)((uint8_t *)cached + dim);
        t->fd = -1;  /* mapped; no descriptor kept */
        return t;
    }

    const js_node *offs = js_get(entry, "data_offsets");
    if (!offs || offs->kind != JS_ARR || offs->n != 2 || offs->kids[0].kind != JS_NUM || offs->kids[1].kind != JS_NUM)
        die("Failed to get data offsets for %s%s", name, "");
    const size_t start = (size_t)offs->kids[0].num, end = (size_t)offs->kids[1].num;
    if (end < start || end > data_bytes || end - start != dim * item) {
        fprintf(stderr, "Data size mismatch for %s: expected %zu, got %zu\n", name, dim * item,
                end >= start ? end - start : 0);
        exit(EXIT_FAILURE);
    }
    Tensor src = {0};
    src.type = src_type;
    src.data = (TensorData *)(data + start);
    src.dim = dim;
    src.vdim = vdim;
    src.hdim = hdim;
    Tensor *result = convert(&src, target);
    if (!result) {
        fprintf(stderr, "Unsupported conversion of tensor %s:  %d -> %d\n", name, (int)src_type, (int)target);
        exit(EXIT_FAILURE);
    }
    if (result == &src) {  /* same type: keep a tensor that points into the (kept) file mapping */
        result = host_calloc(1, sizeof(Tensor));
        *result = src;
        result->fd = -2;  /* not owned: tensor_destroy must not free or unmap it */
    }

    char dir[1024];
    make_dir("cache");
    snprintf(dir, sizeof dir, "cache/%s", model_name);
    make_dir(dir);
    FILE *f = fopen(cache_name, "wb");
    if (!f) die("Failed to open cache file for writing: %s%s", cache_name, "");
    size_t ok = fwrite(result->data, (size_t)quant_size(target), result->dim, f) == result->dim;
    if (result->scale) ok &= fwrite(result->scale, sizeof(float), result->dim / 32, f) == result->dim / 32;
    if (fclose(f) != 0 || !ok) die("Failed to write cache file: %s%s", cache_name, "");
    return result;
}

/* Tensors of one .safetensors file into st; returns how many were taken. */
static int process_file(const char *model_name, const char *path, Model *st) {
    const Config *c = st->config;
    const size_t dim = (size_t)c->dim, hidden = (size_t)c->hidden_dim, vocab = (size_t)c->vocab_size;
    const size_t kv_dim = dim * (size_t)c->n_kv_heads / (size_t)c->n_heads;
    printf("Processing safetensors file: %s\n", path);
    size_t bytes = 0;
    uint8_t *map = map_file(path, &bytes);
    if (!map) {
        fprintf(stderr, "Failed to open safetensors file: %s\n", path);
        return 0;
    }
    uint64_t hlen = 0;
    if (bytes >= 8)
        for (int i = 0; i < 8; ++i) hlen |= (uint64_t)map[i] << (8 * i);
    char err[160] = "";
    js_node *header = (bytes >= 8 && hlen <= bytes - 8) ? js_parse((const char *)map + 8, (size_t)hlen, err, sizeof err)
                                                       : NULL;
    if (!header || header->kind != JS_OBJ) {
        fprintf(stderr, "Skipping %s: not a safetensors file (%s)\n", path, err[0] ? err : "bad header length");
        js_free(header);
        munmap(map, bytes);
        return 0;
    }
    const uint8_t *data = map + 8 + hlen;
    const size_t data_bytes = bytes - 8 - (size_t)hlen;
    int found = 0;
    static const char prefix[] = "model.layers.";
    for (int j = 0; j < header->n; ++j) {
        const char *name = header->keys[j];
        const js_node *e = &header->kids[j];
        Tensor **slot = NULL;
        size_t expect = 0;
        quant_t target = Q8_0;
        if (strcmp(name, "model.embed_tokens.weight") == 0) { slot = &st->token_embedding_table; expect = vocab * dim; }
        else if (strcmp(name, "model.norm.weight") == 0) { slot = &st->rms_final_weight; expect = dim; target = F32; }
        else if (strcmp(name, "lm_head.weight") == 0) { slot = &st->wcls; expect = vocab * dim; }
        else if (strncmp(name, prefix, sizeof prefix - 1) == 0) {
            int layer = -1;
            char comp[256];
            if (sscanf(name + sizeof prefix - 1, "%d.%255s", &layer, comp) != 2 || layer < 0 || layer >= c->n_layers)
                continue;
            Layer *L = &st->layers[layer];
            if (strcmp(comp, "input_layernorm.weight") == 0) { slot = &L->rms_att_weight; expect = dim; target = F32; }
            else if (strcmp(comp, "post_attention_layernorm.weight") == 0) { slot = &L->rms_ffn_weight; expect = dim; target = F32; }
            else if (strcmp(comp, "self_attn.q_proj.weight") == 0) { slot = &L->wq; expect = dim * dim; }
            else if (strcmp(comp, "self_attn.k_proj.weight") == 0) { slot = &L->wk; expect = dim * kv_dim; }
            else if (strcmp(comp, "self_attn.v_proj.weight") == 0) { slot = &L->wv; expect = dim * kv_dim; }
            else if (strcmp(comp, "self_attn.o_proj.weight") == 0) { slot = &L->wo; expect = dim * dim; }
            else if (strcmp(comp, "mlp.gate_proj.weight") == 0) { slot = &L->w1; expect = dim * hidden; }
            else if (strcmp(comp, "mlp.down_proj.weight") == 0) { slot = &L->w2; expect = dim * hidden; }
            else if (strcmp(comp, "mlp.up_proj.weight") == 0) { slot = &L->w3; expect = dim * hidden; }
        }
        if (!slot || *slot) continue;
        *slot = load_tensor(e, model_name, data, data_bytes, name, expect, target);
        found++;
    }
    js_free(header);
    /* The mapping stays: F32 tensors read straight from the file point into it, as in the reference. */
    return found;
}

typedef struct {
    Model model;  /* first: a Model* to the block is a pointer to this member */
    struct dk_model *engine;
    int tp[2];    /* tensor-parallel rank, world of the engine */
} model_ext;

Model *model_ext_alloc(void) { return &((model_ext *)host_calloc(1, sizeof(model_ext)))->model; }

struct dk_model **model_engine_slot(Model *m) { return &((model_ext *)m)->engine; }

int *model_tp_slot(Model *m) { return ((model_ext *)m)->tp; }

static int cmp_names(const void *a, const void *b) { return strcmp(*(char *const *)a, *(char *const *)b); }

static int ends_with(const char *s, const char *suffix) {
    const size_t n = strlen(s), m = strlen(suffix);
    return n >= m && strcmp(s + n - m, suffix) == 0;
}

Model *load_safetensors(const char *dir) {
    const char *slash = strrchr(dir, '/');
    const char *model_name = slash ? slash + 1 : dir;

    char path[4096];
    snprintf(path, sizeof path, "%s/config.json", dir);
    size_t cbytes = 0;
    void *cmap = map_file(path, &cbytes);
    if (!cmap) die("Failed to read %s%s", path, "");
    char err[160] = "";
    js_node *cfg = js_parse((const char *)cmap, cbytes, err, sizeof err);
    munmap(cmap, cbytes);
    if (!cfg || cfg->kind != JS_OBJ) die("Failed to parse %s: %s", path, err);
    Config *config = host_calloc(1, sizeof(Config));
    config->dim = (int)js_num(cfg, "hidden_size", 0);
    config->n_layers = (int)js_num(cfg, "num_hidden_layers", 0);
    config->n_heads = (int)js_num(cfg, "num_attention_heads", 0);
    config->n_kv_heads = (int)js_num(cfg, "num_key_value_heads", 0);
    config->vocab_size = (int)js_num(cfg, "vocab_size", 0);
    config->hidden_dim = (int)js_num(cfg, "intermediate_size", 0);
    config->seq_len = (int)js_num(cfg, "max_position_embeddings", 0);
    js_free(cfg);
    if (config->dim <= 0 || config->n_layers <= 0 || config->n_heads <= 0 || config->n_kv_heads <= 0 ||
        config->vocab_size <= 0 || config->hidden_dim <= 0 || config->seq_len <= 0 || config->dim % config->n_heads)
        die("Bad or incomplete config in %s%s", path, "");

    Model *st = model_ext_alloc();
    st->config = config;
    st->huggingface_rope = true;
    st->layers = host_calloc((size_t)config->n_layers, sizeof(Layer));

    DIR *d = opendir(dir);
    if (!d) die("Failed to open directory: %s%s", dir, "");
    char **files = NULL;
    size_t nfiles = 0, cap = 0;
    for (struct dirent *e; (e = readdir(d)) != NULL;) {
        if (!ends_with(e->d_name, ".safetensors")) continue;
        if (nfiles == cap) {
            cap = cap ? 2 * cap : 16;
            char **nf = realloc(files, cap * sizeof(char *));
            if (!nf) die("out of memory listing %s%s", dir, "");
            files = nf;
        }
        files[nfiles++] = strdup(e->d_name);
    }
    closedir(d);
    qsort(files, nfiles, sizeof(char *), cmp_names);
    int loaded = 0;
    for (size_t i = 0; i < nfiles; ++i) {
        snprintf(path, sizeof path, "%s/%s", dir, files[i]);
        loaded += process_file(model_name, path, st);
        free(files[i]);
    }
    free(files);
    if (loaded == 0) die("No safetensors files found in directory: %s%s", dir, "");
    printf("Loaded %d tensors from safetensors files\n", loaded);
    if (!st->token_embedding_table) die("Missing required tensor: %s%s", "model.embed_tokens.weight", "");
    if (!st->rms_final_weight) die("Missing required tensor: %s%s", "model.norm.weight", "");
    if (!st->wcls) die("Missing required tensor: %s%s", "lm_head.weight", "");
    for (int i = 0; i < config->n_layers; ++i) {
        const Layer *L = &st->layers[i];
        if (!L->rms_att_weight || !L->wq || !L->wk || !L->wv || !L->wo || !L->rms_ffn_weight || !L->w1 || !L->w2 ||
            !L->w3) {
            fprintf(stderr, "Missing required tensor in layer %d\n", i);
            exit(EXIT_FAILURE);
        }
    }
    init_utils(config->dim, config->hidden_dim);
    return st;
}
