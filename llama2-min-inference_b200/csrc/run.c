/*
 * Runner CLI over the llama2q C ABI: the command line, tokenizer, sampler,
 * generate and chat loops of the reference runners (v1-int8-vnni/runq.c:
 * 426-870, GPU form v5-cuda-fused/run.cu:700-1171), driving the B200 decode
 * step.  Same flags and defaults as runq.c (-t 1.0, -p 0.9, -s time, -n 256,
 * -i, -z tokenizer.bin, -m generate|chat, -y), the same tokenizer.bin
 * format and the same "achieved tok/s" line on stderr.  With -t 0 the
 * greedy choice is made on the GPU and only the token id is copied back.
 */
#include <ctype.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "llama2q.h"

/* ---- tokenizer (format and behaviour of runq.c:426-560) ------------------ */

typedef struct {
    char** piece;    /* token strings */
    float* score;    /* merge scores */
    int* order;      /* token ids sorted by string, for binary search */
    int n;
    int max_len;
    char byte_piece[256][2];
} Vocab;

static Vocab* g_sort_vocab; /* qsort has no context argument */

static int cmp_piece(const void* a, const void* b) {
    return strcmp(g_sort_vocab->piece[*(const int*)a], g_sort_vocab->piece[*(const int*)b]);
}

static void die(const char* msg, const char* arg) {
    fprintf(stderr, "%s%s\n", msg, arg ? arg : "");
    exit(EXIT_FAILURE);
}

static void vocab_load(Vocab* v, const char* path, int n) {
    FILE* f = fopen(path, "rb");
    if (!f) die("couldn't load ", path);
    v->n = n;
    v->piece = (char**)calloc((size_t)n, sizeof(char*));
    v->score = (float*)calloc((size_t)n, sizeof(float));
    v->order = NULL;
    for (int i = 0; i < 256; i++) {
        v->byte_piece[i][0] = (char)i;
        v->byte_piece[i][1] = '\0';
    }
    if (fread(&v->max_len, sizeof(int), 1, f) != 1) die("failed read", NULL);
    for (int i = 0; i < n; i++) {
        int len;
        if (fread(&v->score[i], sizeof(float), 1, f) != 1 || fread(&len, sizeof(int), 1, f) != 1)
            die("failed read", NULL);
        v->piece[i] = (char*)malloc((size_t)len + 1);
        if (len > 0 && fread(v->piece[i], (size_t)len, 1, f) != 1) die("failed read", NULL);
        v->piece[i][len] = '\0';
    }
    fclose(f);
}

static void vocab_free(Vocab* v) {
    for (int i = 0; i < v->n; i++) free(v->piece[i]);
    free(v->piece);
    free(v->score);
    free(v->order);
}

static int vocab_find(Vocab* v, const char* s) {
    int lo = 0, hi = v->n - 1;
    while (lo <= hi) {
        int mid = (lo + hi) / 2;
        int c = strcmp(s, v->piece[v->order[mid]]);
        if (c == 0) return v->order[mid];
        if (c < 0) hi = mid - 1;
        else lo = mid + 1;
    }
    return -1;
}

/* piece printed after `prev`: a leading space is dropped after BOS, and
 * <0xXX> pieces become raw bytes */
static const char* vocab_decode(Vocab* v, int prev, int tok) {
    const char* p = v->piece[tok];
    if (prev == 1 && p[0] == ' ') p++;
    unsigned char b;
    if (sscanf(p, "<0x%02hhX>", &b) == 1) p = v->byte_piece[b];
    return p;
}

static void print_piece(const char* p) {
    if (!p || !p[0]) return;
    if (!p[1] && !(isprint((unsigned char)p[0]) || isspace((unsigned char)p[0]))) return;
    printf("%s", p);
}

/* UTF-8 code points to tokens (byte fallback = byte + 3), then repeatedly
 * merge the adjacent pair whose concatenation has the best score */
static void vocab_encode(Vocab* v, const char* text, int bos, int eos, int* out, int* n_out) {
    if (!v->order) {
        v->order = (int*)malloc(sizeof(int) * (size_t)v->n);
        for (int i = 0; i < v->n; i++) v->order[i] = i;
        g_sort_vocab = v;
        qsort(v->order, (size_t)v->n, sizeof(int), cmp_piece);
    }
    char* buf = (char*)malloc((size_t)v->max_len * 2 + 3);
    int n = 0;
    if (bos) out[n++] = 1;
    if (text[0]) out[n++] = vocab_find(v, " ");
    size_t len = 0;
    for (const char* c = text; *c; c++) {
        if ((*c & 0xC0) != 0x80) len = 0;
        buf[len++] = *c;
        buf[len] = '\0';
        if ((c[1] & 0xC0) == 0x80 && len < 4) continue;
        int id = vocab_find(v, buf);
        if (id >= 0) {
            out[n++] = id;
        } else {
            for (size_t i = 0; i < len; i++) out[n++] = (unsigned char)buf[i] + 3;
        }
        len = 0;
    }
    for (;;) {
        float best = -1e10f;
        int best_id = -1, at = -1;
        for (int i = 0; i + 1 < n; i++) {
            snprintf(buf, (size_t)v->max_len * 2 + 3, "%s%s", v->piece[out[i]], v->piece[out[i + 1]]);
            int id = vocab_find(v, buf);
            if (id >= 0 && v->score[id] > best) {
                best = v->score[id];
                best_id = id;
                at = i;
            }
        }
        if (at < 0) break;
        out[at] = best_id;
        memmove(out + at + 1, out + at + 2, sizeof(int) * (size_t)(n - at - 2));
        n--;
    }
    if (eos) out[n++] = 2;
    free(buf);
    *n_out = n;
}

/* ---- sampler (behaviour of runq.c:565-667) ----------------------------- */

typedef struct {
    float p;
    int i;
} Cand;

typedef struct {
    int n;
    float temperature, topp;
    unsigned long long rng;
    Cand* cand;
} Sampler;

static unsigned int rng_u32(unsigned long long* s) { /* xorshift64* */
    *s ^= *s >> 12;
    *s ^= *s << 25;
    *s ^= *s >> 27;
    return (unsigned int)((*s * 0x2545F4914F6CDD1Dull) >> 32);
}

static float rng_f32(unsigned long long* s) { return (float)(rng_u32(s) >> 8) / 16777216.0f; }

static void softmax_host(float* x, int n) {
    float m = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > m) m = x[i];
    float s = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - m);
        s += x[i];
    }
    for (int i = 0; i < n; i++) x[i] /= s;
}

static int cmp_cand(const void* a, const void* b) {
    float pa = ((const Cand*)a)->p, pb = ((const Cand*)b)->p;
    return pa > pb ? -1 : (pa < pb ? 1 : 0);
}

static int sample_logits(Sampler* s, float* logits) {
    for (int i = 0; i < s->n; i++) logits[i] /= s->temperature;
    softmax_host(logits, s->n);
    float coin = rng_f32(&s->rng);
    if (s->topp <= 0 || s->topp >= 1) {
        float cdf = 0.0f;
        for (int i = 0; i < s->n; i++) {
            cdf += logits[i];
            if (coin < cdf) return i;
        }
        return s->n - 1;
    }
    /* top-p: drop tokens that cannot be in the nucleus, sort the rest */
    const float cutoff = (1.0f - s->topp) / (float)(s->n - 1);
    int m = 0;
    for (int i = 0; i < s->n; i++)
        if (logits[i] >= cutoff) {
            s->cand[m].i = i;
            s->cand[m].p = logits[i];
            m++;
        }
    qsort(s->cand, (size_t)m, sizeof(Cand), cmp_cand);
    float cum = 0.0f;
    int last = m - 1;
    for (int i = 0; i < m; i++) {
        cum += s->cand[i].p;
        if (cum > s->topp) {
            last = i;
            break;
        }
    }
    float r = coin * cum, cdf = 0.0f;
    for (int i = 0; i <= last; i++) {
        cdf += s->cand[i].p;
        if (r < cdf) return s->cand[i].i;
    }
    return s->cand[last].i;
}

/* first index of the maximum (sample_argmax, runq.c:578-585) */
static int argmax_first(const float* x, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return best;
}

/* next token after a forward step at (token, pos) */
static int step(Transformer* t, Sampler* s, int token, int pos, int sample) {
    if (!sample) {
        /* prompt token: logits are not needed, still run the step */
        int dummy;
        if (forward_argmax(t, token, pos, &dummy) != LQ_OK) die("forward failed: ", lq_last_error());
        return -1;
    }
    if (s->temperature == 0.0f) {
        int nxt;
        if (forward_argmax(t, token, pos, &nxt) != LQ_OK) die("forward failed: ", lq_last_error());
        return nxt;
    }
    float* logits = forward(t, token, pos);
    if (!logits) die("forward failed: ", lq_last_error());
    return sample_logits(s, logits);
}

static long now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_REALTIME, &ts);
    return ts.tv_sec * 1000 + ts.tv_nsec / 1000000;
}

/* ---- loops (runq.c:681-794) -------------------------------------------- */

static void generate(Transformer* t, Vocab* v, Sampler* s, const char* prompt, int steps) {
    if (!prompt) prompt = "";
    int* toks = (int*)malloc(sizeof(int) * (strlen(prompt) + 3));
    int np = 0;
    vocab_encode(v, prompt, 1, 0, toks, &np);
    if (np < 1) die("something is wrong, expected at least 1 prompt token", NULL);
    long start = 0;
    int token = toks[0], pos = 0, timed0 = 1; /* steps timed: those after the first forward call */
    if (np >= 2 && steps >= np) {
        /* the whole prompt in one prefill call (rows of one sequence through
         * every product together), then sample from its last token's logits:
         * the same tokens and printed pieces as feeding it one at a time */
        float* logits = forward_prompt(t, toks, np, 0);
        if (!logits) die("forward failed: ", lq_last_error());
        for (int i = 0; i + 1 < np; ++i) print_piece(vocab_decode(v, toks[i], toks[i + 1]));
        fflush(stdout);
        const int next = s->temperature == 0.0f ? argmax_first(logits, v->n) : sample_logits(s, logits);
        token = toks[np - 1];
        pos = np;
        start = now_ms();
        timed0 = np;
        if (next == 1) {
            printf("\n");
            free(toks);
            return;
        }
        print_piece(vocab_decode(v, token, next));
        fflush(stdout);
        token = next;
    }
    while (pos < steps) {
        int in_prompt = pos < np - 1;
        int next = step(t, s, token, pos, !in_prompt);
        if (in_prompt) next = toks[pos + 1];
        pos++;
        if (next == 1) break;
        print_piece(vocab_decode(v, token, next));
        fflush(stdout);
        token = next;
        if (start == 0) start = now_ms();
    }
    printf("\n");
    if (pos > timed0) fprintf(stderr, "achieved tok/s: %f\n", (pos - timed0) / (double)(now_ms() - start) * 1000);
    free(toks);
}

static int read_line(const char* guide, char* buf, size_t size) {
    printf("%s", guide);
    if (!fgets(buf, (int)size, stdin)) return 0;
    size_t n = strlen(buf);
    if (n && buf[n - 1] == '\n') buf[n - 1] = '\0';
    return 1;
}

static void chat(Transformer* t, Vocab* v, Sampler* s, const char* user0, const char* sys0, int steps) {
    char sys_prompt[512] = "", user[512] = "", rendered[1152];
    int* toks = (int*)malloc(sizeof(int) * 1152);
    int np = 0, idx = 0, user_turn = 1, next = 0, token, pos = 0;
    while (pos < steps) {
        if (user_turn) {
            if (pos == 0) {
                if (sys0) snprintf(sys_prompt, sizeof(sys_prompt), "%s", sys0);
                else read_line("Enter system prompt (optional): ", sys_prompt, sizeof(sys_prompt));
            }
            if (pos == 0 && user0) snprintf(user, sizeof(user), "%s", user0);
            else if (!read_line("User: ", user, sizeof(user))) break;
            if (pos == 0 && sys_prompt[0])
                snprintf(rendered, sizeof(rendered), "[INST] <<SYS>>\n%s\n<</SYS>>\n\n%s [/INST]", sys_prompt, user);
            else
                snprintf(rendered, sizeof(rendered), "[INST] %s [/INST]", user);
            vocab_encode(v, rendered, 1, 0, toks, &np);
            idx = 0;
            user_turn = 0;
            printf("Assistant: ");
        }
        token = idx < np ? toks[idx++] : next;
        if (token == 2) user_turn = 1;
        next = step(t, s, token, pos, 1);
        pos++;
        if (idx >= np && next != 2) {
            print_piece(vocab_decode(v, token, next));
            fflush(stdout);
        }
        if (next == 2) printf("\n");
    }
    printf("\n");
    free(toks);
}

static void usage(void) {
    fprintf(stderr, "Usage:   run <checkpoint> [options]\n");
    fprintf(stderr, "Example: run llama2-7b-q4.bin -n 256 -i \"Once upon a time\"\n");
    fprintf(stderr, "Options:\n");
    fprintf(stderr, "  -t <float>  temperature in [0,inf], default 1.0\n");
    fprintf(stderr, "  -p <float>  p value in top-p (nucleus) sampling in [0,1] default 0.9\n");
    fprintf(stderr, "  -s <int>    random seed, default time(NULL)\n");
    fprintf(stderr, "  -n <int>    number of steps to run for, default 256. 0 = max_seq_len\n");
    fprintf(stderr, "  -i <string> input prompt\n");
    fprintf(stderr, "  -z <string> optional path to custom tokenizer\n");
    fprintf(stderr, "  -m <string> mode: generate|chat, default: generate\n");
    fprintf(stderr, "  -y <string> (optional) system prompt in chat mode\n");
    exit(EXIT_FAILURE);
}

int main(int argc, char** argv) {
    const char *ckpt = NULL, *tok_path = "tokenizer.bin", *prompt = NULL, *mode = "generate", *sys_prompt = NULL;
    float temperature = 1.0f, topp = 0.9f;
    int steps = 256;
    unsigned long long seed = 0;
    if (argc < 2) usage();
    ckpt = argv[1];
    for (int i = 2; i < argc; i += 2) {
        if (i + 1 >= argc || argv[i][0] != '-' || strlen(argv[i]) != 2) usage();
        const char* val = argv[i + 1];
        switch (argv[i][1]) {
            case 't': temperature = (float)atof(val); break;
            case 'p': topp = (float)atof(val); break;
            case 's': seed = (unsigned long long)atoi(val); break;
            case 'n': steps = atoi(val); break;
            case 'i': prompt = val; break;
            case 'z': tok_path = val; break;
            case 'm': mode = val; break;
            case 'y': sys_prompt = val; break;
            default: usage();
        }
    }
    if (seed <= 0) seed = (unsigned int)time(NULL);
    if (temperature < 0.0f) temperature = 0.0f;
    if (topp < 0.0f || topp > 1.0f) topp = 0.9f;
    if (steps < 0) steps = 0;
    if (lq_select_device(-1) != LQ_OK) die("no CUDA device: ", lq_last_error());

    Transformer* t = NULL;
    if (build_transformer(&t, ckpt, 0) != LQ_OK) die("", lq_last_error());
    Config cfg;
    transformer_config(t, &cfg, NULL, NULL);
    if (steps == 0 || steps > cfg.seq_len) steps = cfg.seq_len;
    Vocab v;
    vocab_load(&v, tok_path, cfg.vocab_size);
    Sampler s = {cfg.vocab_size, temperature, topp, seed, (Cand*)malloc(sizeof(Cand) * (size_t)cfg.vocab_size)};
    if (strcmp(mode, "generate") == 0) {
        generate(t, &v, &s, prompt, steps);
    } else if (strcmp(mode, "chat") == 0) {
        chat(t, &v, &s, prompt, sys_prompt, steps);
    } else {
        fprintf(stderr, "unknown mode: %s\n", mode);
        usage();
    }
    free(s.cand);
    vocab_free(&v);
    free_transformer(t);
    return 0;
}
