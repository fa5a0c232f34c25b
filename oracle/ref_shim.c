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
