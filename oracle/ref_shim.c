/*
 * ref_shim.c — plain-pointer wrappers around the reference's own dequant
 * entry points, so the unmodified engine/src/gguf.c (compiled from the
 * reference tree into oracle/_ref/) can be called by the parity tests and by
 * the CPU baseline. TEST INFRASTRUCTURE ONLY.
 *
 * gguf_dequantize_tensor_from_buf / gguf_dequantize_expert_slice_from_buf
 * (engine/src/gguf.h:116-127) take a gguf_tensor_info (engine/src/gguf.h:15-23);
 * these wrappers fill one from (type, dims) the way gguf.c's parser would.
 */
#include <string.h>
#include "gguf.h" /* the reference's header, from its own tree (-I) */

int ref_dequant_tensor(const void *data, int type, uint64_t n_elems, float *out) {
    gguf_tensor_info ti;
    memset(&ti, 0, sizeof(ti));
    ti.name = "t";
    ti.type = (ggml_type)type;
    ti.n_dims = 1;
    ti.dims[0] = n_elems;
    ti.n_elems = n_elems;
    ti.size_bytes = ggml_row_size((ggml_type)type, n_elems);
    return gguf_dequantize_tensor_from_buf(data, &ti, out) ? 1 : 0;
}

/* dims = [n_elems/n_experts, n_experts]: the expert dimension is last
 * (fastest-varying in the reference's slice convention). */
int ref_dequant_slice(const void *data, int type, uint64_t n_elems, uint64_t n_experts,
                      int expert, float *out) {
    gguf_tensor_info ti;
    memset(&ti, 0, sizeof(ti));
    ti.name = "t";
    ti.type = (ggml_type)type;
    ti.n_dims = 2;
    ti.dims[0] = n_experts ? n_elems / n_experts : 0;
    ti.dims[1] = n_experts;
    ti.n_elems = n_elems;
    ti.size_bytes = ggml_row_size((ggml_type)type, n_elems);
    return gguf_dequantize_expert_slice_from_buf(data, &ti, expert, out) ? 1 : 0;
}

/* The reference's own GGUF parser on a file: a tensor's type, dims, absolute
 * byte size and bytes (gguf_open / gguf_find_tensor / gguf_read_tensor_data,
 * engine/src/gguf.c),
 * and an architecture-prefixed u32 parameter (gguf_get_param_u32). Returns 1
 * when found. */
int ref_gguf_tensor(const char *path, const char *name, int *type, uint64_t dims[4], void *buf,
                    uint64_t buf_size, uint64_t *size) {
    char err[256];
    gguf_model *m = gguf_open(path, err, sizeof(err));
    if (!m) return 0;
    const gguf_tensor_info *t = gguf_find_tensor(m, name);
    int ok = 0;
    if (t) {
        *type = (int)t->type;
        for (int d = 0; d < 4; d++) dims[d] = t->dims[d];
        *size = (uint64_t)t->size_bytes;
        ok = 1;
        if (buf && buf_size >= t->size_bytes)
            ok = gguf_read_tensor_data(m, t, buf, (size_t)buf_size) == t->size_bytes;
    }
    gguf_close(m);
    return ok;
}

int ref_gguf_u32(const char *path, const char *param, uint32_t *v) {
    char err[256];
    gguf_model *m = gguf_open(path, err, sizeof(err));
    if (!m) return 0;
    int ok = gguf_get_param_u32(m, param, v) ? 1 : 0;
    gguf_close(m);
    return ok;
}
