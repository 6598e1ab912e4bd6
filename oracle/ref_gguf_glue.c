/* ref_gguf_glue.c -- test infrastructure only: a flat C entry point over the
 * reference's own GGUF reader (gguf.c, compiled unmodified from where it
 * lies), so that tests can check, on a GGUF file written by gguf-py, the
 * tensor bytes that a host would hand to moe_load_layer: it reads the stacked
 * expert tensors blk.L.ffn_{gate,up,down}_exps.weight the way infer.m does
 * (gguf_load_manifest, gguf_find, gguf_tensor_pread; gguf.h:168-192). */
#include <stdint.h>
#include <string.h>

#include "gguf.h"

/* Finds `name` in the file at `path`; returns its dims, ggml type and byte
 * size, and reads up to buf_size bytes of it into buf (buf may be NULL).
 * Returns 0 on success, -1 if the file does not load, -2 if the tensor is
 * absent, -3 if the read fails. */
int ref_gguf_tensor(const char *path, const char *name, uint64_t *dims, uint32_t *n_dims, int *type,
                    uint64_t *nbytes, void *buf, uint64_t buf_size) {
    gguf_manifest m;
    memset(&m, 0, sizeof(m));
    const char *paths[1] = {path};
    if (gguf_load_manifest(&m, paths, 1) != 0) return -1;
    const gguf_tensor *t = gguf_find(&m, name);
    if (!t) {
        gguf_free_manifest(&m);
        return -2;
    }
    for (uint32_t i = 0; i < 4; i++) dims[i] = i < t->n_dims ? t->dims[i] : 1;
    *n_dims = t->n_dims;
    *type = (int)t->type;
    *nbytes = t->nbytes;
    int rc = 0;
    if (buf) {
        const uint64_t n = buf_size < t->nbytes ? buf_size : t->nbytes;
        if (gguf_tensor_pread(t, buf, n, 0) != (int64_t)n) rc = -3;
    }
    gguf_free_manifest(&m);
    return rc;
}
