/* host_gguf.c -- a C host of the reference's kind driving libmoe_cuda.so from
 * a GGUF file.  It opens the file with the reference's own reader (gguf.c:
 * gguf_load_manifest / gguf_find / gguf_tensor_pread, gguf.h:168-192), reads
 * one MoE layer's tensors under the names infer.m uses (infer.m:297-305:
 * blk.L.ffn_{gate,up,down}_exps.weight, blk.L.ffn_gate_inp.weight,
 * blk.L.exp_probs_b.bias, blk.L.ffn_{gate,up,down}_shexp.weight) -- of the
 * stacked expert tensors only the rank's slice (moe_shard_range) -- hands
 * them to moe_load_layer_shard and runs moe_forward on the tokens of a raw
 * fp32 file.
 *
 *   host_gguf <file.gguf> <layer> <hidden> <intermediate> <n_experts> <n_group>
 *             <topk_group> <top_k> <tokens.f32> <n_tokens> <out prefix>
 *
 * Writes <prefix>.out (fp32 [n_tokens x hidden]), <prefix>.idx (int32
 * [n_tokens x top_k]) and <prefix>.w (fp32).  Exit status 0 on success. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gguf.h"
#include "moe_cuda.h"

static void *read_tensor(const gguf_manifest *m, const char *fmt, int L, const gguf_tensor **out) {
    char name[256];
    snprintf(name, sizeof(name), fmt, L);
    const gguf_tensor *t = gguf_find(m, name);
    if (!t) {
        fprintf(stderr, "[host] ERROR: tensor %s not found\n", name);
        return NULL;
    }
    void *buf = malloc(t->nbytes);
    if (!buf || gguf_tensor_pread(t, buf, t->nbytes, 0) != (int64_t)t->nbytes) {
        fprintf(stderr, "[host] ERROR: cannot read %s\n", name);
        free(buf);
        return NULL;
    }
    if (out) *out = t;
    return buf;
}

/* The rank's slice of a stacked expert tensor (ne2 = n_experts experts):
 * moe_shard_range gives its byte range, gguf_tensor_pread reads just that
 * (gguf.h:192, `rel` = the offset inside the tensor). */
static void *read_expert_slice(const gguf_manifest *m, const char *fmt, int L, const moe_ctx *moe, int n_experts,
                               const gguf_tensor **out) {
    char name[256];
    snprintf(name, sizeof(name), fmt, L);
    const gguf_tensor *t = gguf_find(m, name);
    if (!t || t->nbytes % (uint64_t)n_experts) {
        fprintf(stderr, "[host] ERROR: tensor %s missing or not %d experts\n", name, n_experts);
        return NULL;
    }
    size_t off = 0, bytes = 0;
    if (moe_shard_range(moe, (size_t)(t->nbytes / (uint64_t)n_experts), &off, &bytes) != 0) return NULL;
    void *buf = malloc(bytes);
    if (!buf || gguf_tensor_pread(t, buf, bytes, off) != (int64_t)bytes) {
        fprintf(stderr, "[host] ERROR: cannot read the expert slice of %s\n", name);
        free(buf);
        return NULL;
    }
    if (out) *out = t;
    return buf;
}

static int write_file(const char *prefix, const char *ext, const void *p, size_t n) {
    char path[1024];
    snprintf(path, sizeof(path), "%s.%s", prefix, ext);
    FILE *f = fopen(path, "wb");
    if (!f || fwrite(p, 1, n, f) != n) {
        fprintf(stderr, "[host] ERROR: cannot write %s\n", path);
        if (f) fclose(f);
        return -1;
    }
    fclose(f);
    return 0;
}

int main(int argc, char **argv) {
    if (argc != 12) {
        fprintf(stderr, "usage: %s file.gguf layer hidden intermediate n_experts n_group topk_group top_k "
                        "tokens.f32 n_tokens out_prefix\n", argv[0]);
        return 2;
    }
    const int L = atoi(argv[2]), T = atoi(argv[10]);
    moe_config cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.hidden = atoi(argv[3]);
    cfg.intermediate = atoi(argv[4]);
    cfg.n_experts = atoi(argv[5]);
    cfg.n_group = atoi(argv[6]);
    cfg.topk_group = atoi(argv[7]);
    cfg.top_k = atoi(argv[8]);
    cfg.routed_scale = 2.5f;
    cfg.rms_eps = 1e-6f;
    cfg.n_layers = 1;
    cfg.max_tokens = T;

    gguf_manifest m;
    memset(&m, 0, sizeof(m));
    const char *paths[1] = {argv[1]};
    if (gguf_load_manifest(&m, paths, 1) != 0) {
        fprintf(stderr, "[host] ERROR: cannot load %s\n", argv[1]);
        return 1;
    }
    const gguf_tensor *tg = NULL, *tu = NULL, *td = NULL, *tr = NULL, *tb = NULL, *tsg = NULL, *tsu = NULL,
                      *tsd = NULL;
    int rc = 1;
    float *h = NULL, *out = NULL, *w = NULL;
    int *idx = NULL;
    void *g = NULL, *u = NULL, *d = NULL;
    /* a rank's context first: it says which experts (bytes) this rank reads */
    moe_ctx *moe = moe_create(&cfg, 0, 0, 1, NULL);
    void *router = read_tensor(&m, "blk.%d.ffn_gate_inp.weight", L, &tr);
    void *bias = read_tensor(&m, "blk.%d.exp_probs_b.bias", L, &tb);
    void *sg = read_tensor(&m, "blk.%d.ffn_gate_shexp.weight", L, &tsg);
    void *su = read_tensor(&m, "blk.%d.ffn_up_shexp.weight", L, &tsu);
    void *sd = read_tensor(&m, "blk.%d.ffn_down_shexp.weight", L, &tsd);
    if (!moe) goto done;
    g = read_expert_slice(&m, "blk.%d.ffn_gate_exps.weight", L, moe, cfg.n_experts, &tg);
    u = read_expert_slice(&m, "blk.%d.ffn_up_exps.weight", L, moe, cfg.n_experts, &tu);
    d = read_expert_slice(&m, "blk.%d.ffn_down_exps.weight", L, moe, cfg.n_experts, &td);
    if (!g || !u || !d || !router || !bias || !sg || !su || !sd) goto done;
    if (tr->type != 0 || tb->type != 0) {  /* GGML_TYPE_F32 */
        fprintf(stderr, "[host] ERROR: router and bias must be F32\n");
        goto done;
    }
    /* the layer goes into slot 0 of this one-layer context */
    if (moe_load_layer_shard(moe, 0, g, u, d, (int)td->type, (const float *)router, (const float *)bias, sg, su,
                             sd, (int)tsd->type) != 0) {
        fprintf(stderr, "[host] ERROR: %s\n", moe_last_error(moe));
        goto done;
    }
    const size_t nh = (size_t)T * cfg.hidden, nk = (size_t)T * cfg.top_k;
    h = malloc(nh * sizeof(float));
    out = malloc(nh * sizeof(float));
    idx = malloc(nk * sizeof(int));
    w = malloc(nk * sizeof(float));
    FILE *f = fopen(argv[9], "rb");
    if (!f || fread(h, sizeof(float), nh, f) != nh) {
        fprintf(stderr, "[host] ERROR: cannot read %d tokens from %s\n", T, argv[9]);
        if (f) fclose(f);
        goto done;
    }
    fclose(f);
    if (moe_forward(moe, 0, h, T, out, idx, w) != 0) {
        fprintf(stderr, "[host] ERROR: %s\n", moe_last_error(moe));
        goto done;
    }
    if (write_file(argv[11], "out", out, nh * sizeof(float)) || write_file(argv[11], "idx", idx, nk * sizeof(int)) ||
        write_file(argv[11], "w", w, nk * sizeof(float)))
        goto done;
    rc = 0;
done:
    moe_destroy(moe);
    free(g); free(u); free(d); free(router); free(bias); free(sg); free(su); free(sd);
    free(h); free(out); free(idx); free(w);
    gguf_free_manifest(&m);
    return rc;
}
