/*
 * json.c -- the JSON subset the loader needs: the safetensors header (an object of objects holding
 * strings, numbers and arrays of numbers) and HF config.json.  Recursive descent over a bounded
 * buffer (no NUL terminator needed), depth-limited, strings decoded to UTF-8 with \uXXXX escapes
 * and surrogate pairs.  Replaces the reference's use of the parson library (src/parson.c) for
 * json_parse_string / json_parse_file / json_object_get_* (src/safetensors.c:160-166, :290-300).
 */
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "host_internal.h"

enum { kMaxDepth = 64 };

typedef struct {
    const char *p, *end;
    char *err;
    size_t err_len;
    int failed;
} js_parser;

static void js_fail(js_parser *ps, const char *what) {
    if (!ps->failed && ps->err && ps->err_len)
        snprintf(ps->err, ps->err_len, "JSON: %s at byte %ld", what, (long)(ps->end - ps->p));
    ps->failed = 1;
}

static void js_ws(js_parser *ps) {
    while (ps->p < ps->end && (*ps->p == ' ' || *ps->p == '\t' || *ps->p == '\n' || *ps->p == '\r')) ps->p++;
}

static int js_hex4(js_parser *ps, unsigned *out) {
    if (ps->end - ps->p < 4) return 0;
    unsigned v = 0;
    for (int i = 0; i < 4; ++i) {
        const char c = ps->p[i];
        v <<= 4;
        if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
        else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
        else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
        else return 0;
    }
    ps->p += 4;
    *out = v;
    return 1;
}

static size_t js_utf8(unsigned cp, char *o) {
    if (cp < 0x80) { o[0] = (char)cp; return 1; }
    if (cp < 0x800) { o[0] = (char)(0xC0 | (cp >> 6)); o[1] = (char)(0x80 | (cp & 0x3F)); return 2; }
    if (cp < 0x10000) {
        o[0] = (char)(0xE0 | (cp >> 12)); o[1] = (char)(0x80 | ((cp >> 6) & 0x3F)); o[2] = (char)(0x80 | (cp & 0x3F));
        return 3;
    }
    o[0] = (char)(0xF0 | (cp >> 18)); o[1] = (char)(0x80 | ((cp >> 12) & 0x3F));
    o[2] = (char)(0x80 | ((cp >> 6) & 0x3F)); o[3] = (char)(0x80 | (cp & 0x3F));
    return 4;
}

/* At an opening quote: returns the decoded string (malloc'd) or NULL. */
static char *js_string(js_parser *ps) {
    ps->p++;  /* the quote */
    const char *start = ps->p;
    /* The decoded string is never longer than the escaped one. */
    while (ps->p < ps->end && *ps->p != '"') ps->p += (*ps->p == '\\' && ps->p + 1 < ps->end) ? 2 : 1;
    if (ps->p >= ps->end) { js_fail(ps, "unterminated string"); return NULL; }
    const size_t raw = (size_t)(ps->p - start);
    char *out = malloc(raw + 1);
    if (!out) { js_fail(ps, "out of memory"); return NULL; }
    js_parser sub = {start, ps->p, ps->err, ps->err_len, 0};
    size_t k = 0;
    while (sub.p < sub.end) {
        char c = *sub.p++;
        if ((unsigned char)c < 0x20) { free(out); js_fail(ps, "control character in string"); return NULL; }
        if (c != '\\') { out[k++] = c; continue; }
        c = *sub.p++;
        switch (c) {
            case '"': out[k++] = '"'; break;
            case '\\': out[k++] = '\\'; break;
            case '/': out[k++] = '/'; break;
            case 'b': out[k++] = '\b'; break;
            case 'f': out[k++] = '\f'; break;
            case 'n': out[k++] = '\n'; break;
            case 'r': out[k++] = '\r'; break;
            case 't': out[k++] = '\t'; break;
            case 'u': {
                unsigned cp;
                if (!js_hex4(&sub, &cp)) { free(out); js_fail(ps, "bad \\u escape"); return NULL; }
                if (cp >= 0xD800 && cp < 0xDC00) {  /* high surrogate: a low one must follow */
                    unsigned lo;
                    if (sub.end - sub.p < 6 || sub.p[0] != '\\' || sub.p[1] != 'u') {
                        free(out); js_fail(ps, "lone surrogate"); return NULL;
                    }
                    sub.p += 2;
                    if (!js_hex4(&sub, &lo) || lo < 0xDC00 || lo >= 0xE000) {
                        free(out); js_fail(ps, "bad surrogate pair"); return NULL;
                    }
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                } else if (cp >= 0xDC00 && cp < 0xE000) {
                    free(out); js_fail(ps, "lone surrogate"); return NULL;
                }
                k += js_utf8(cp, out + k);  /* <= 4 bytes from >= 6 escaped ones */
                break;
            }
            default: free(out); js_fail(ps, "bad escape"); return NULL;
        }
    }
    out[k] = '\0';
    ps->p++;  /* closing quote */
    return out;
}

static int js_value(js_parser *ps, js_node *v, int depth);

static int js_push(js_node *v, int *cap) {
    if (v->n < *cap) return 1;
    const int nc = *cap ? 2 * *cap : 8;
    js_node *kids = realloc(v->kids, (size_t)nc * sizeof(js_node));
    if (!kids) return 0;
    v->kids = kids;
    if (v->kind == JS_OBJ) {
        char **keys = realloc(v->keys, (size_t)nc * sizeof(char *));
        if (!keys) return 0;
        v->keys = keys;
    }
    *cap = nc;
    return 1;
}

static int js_container(js_parser *ps, js_node *v, int depth, int is_obj) {
    v->kind = is_obj ? JS_OBJ : JS_ARR;
    ps->p++;
    int cap = 0;
    js_ws(ps);
    if (ps->p < ps->end && *ps->p == (is_obj ? '}' : ']')) { ps->p++; return 1; }
    for (;;) {
        js_ws(ps);
        char *key = NULL;
        if (is_obj) {
            if (ps->p >= ps->end || *ps->p != '"') { js_fail(ps, "expected a member name"); return 0; }
            if (!(key = js_string(ps))) return 0;
            js_ws(ps);
            if (ps->p >= ps->end || *ps->p != ':') { free(key); js_fail(ps, "expected ':'"); return 0; }
            ps->p++;
        }
        if (!js_push(v, &cap)) { free(key); js_fail(ps, "out of memory"); return 0; }
        js_node *kid = &v->kids[v->n];
        memset(kid, 0, sizeof(*kid));
        if (is_obj) v->keys[v->n] = key;
        v->n++;
        if (!js_value(ps, kid, depth + 1)) return 0;
        js_ws(ps);
        if (ps->p < ps->end && *ps->p == ',') { ps->p++; continue; }
        if (ps->p < ps->end && *ps->p == (is_obj ? '}' : ']')) { ps->p++; return 1; }
        js_fail(ps, is_obj ? "expected ',' or '}'" : "expected ',' or ']'");
        return 0;
    }
}

static int js_literal(js_parser *ps, const char *word) {
    const size_t n = strlen(word);
    if ((size_t)(ps->end - ps->p) < n || memcmp(ps->p, word, n) != 0) return 0;
    ps->p += n;
    return 1;
}

static int js_value(js_parser *ps, js_node *v, int depth) {
    if (depth > kMaxDepth) { js_fail(ps, "nesting too deep"); return 0; }
    js_ws(ps);
    if (ps->p >= ps->end) { js_fail(ps, "unexpected end"); return 0; }
    const char c = *ps->p;
    if (c == '{' || c == '[') return js_container(ps, v, depth, c == '{');
    if (c == '"') {
        v->kind = JS_STR;
        return (v->str = js_string(ps)) != NULL;
    }
    if (js_literal(ps, "true")) { v->kind = JS_BOOL; v->num = 1; return 1; }
    if (js_literal(ps, "false")) { v->kind = JS_BOOL; v->num = 0; return 1; }
    if (js_literal(ps, "null")) { v->kind = JS_NULL; return 1; }
    if (c == '-' || (c >= '0' && c <= '9')) {
        char buf[64];
        size_t k = 0;
        while (ps->p + k < ps->end && k < sizeof(buf) - 1 && strchr("+-.eE0123456789", ps->p[k])) {
            buf[k] = ps->p[k];
            k++;
        }
        buf[k] = '\0';
        char *stop = NULL;
        errno = 0;
        v->num = strtod(buf, &stop);
        if (stop == buf || (size_t)(stop - buf) != k) { js_fail(ps, "bad number"); return 0; }
        v->kind = JS_NUM;
        ps->p += k;
        return 1;
    }
    js_fail(ps, "unexpected character");
    return 0;
}

static void js_clear(js_node *v) {
    if (v->kind == JS_STR) free(v->str);
    if (v->kind == JS_ARR || v->kind == JS_OBJ) {
        for (int i = 0; i < v->n; ++i) {
            js_clear(&v->kids[i]);
            if (v->kind == JS_OBJ) free(v->keys[i]);
        }
        free(v->kids);
        free(v->keys);
    }
}

void js_free(js_node *v) {
    if (!v) return;
    js_clear(v);
    free(v);
}

js_node *js_parse(const char *text, size_t len, char *err, size_t err_len) {
    js_parser ps = {text, text + len, err, err_len, 0};
    js_node *v = calloc(1, sizeof(js_node));
    if (!v) return NULL;
    if (!js_value(&ps, v, 0)) { js_free(v); return NULL; }
    js_ws(&ps);
    if (ps.p != ps.end) {
        js_fail(&ps, "trailing characters");
        js_free(v);
        return NULL;
    }
    return v;
}

const js_node *js_get(const js_node *obj, const char *key) {
    if (!obj || obj->kind != JS_OBJ) return NULL;
    for (int i = 0; i < obj->n; ++i)
        if (strcmp(obj->keys[i], key) == 0) return &obj->kids[i];
    return NULL;
}

double js_num(const js_node *obj, const char *key, double dflt) {
    const js_node *v = js_get(obj, key);
    return v && v->kind == JS_NUM ? v->num : dflt;
}
