// Minimal ggml-API shim used only to build the reference's own sources as the
// CPU oracle (test infrastructure, never shipped, never on the product path).
//
// ggml itself is a third-party dependency of the reference that is absent here
// (the `third_party/ggml` submodule is empty and no commit is pinned, see the
// reference's .gitmodules:1-3).  This header declares exactly the symbols the
// reference uses (src/ggml_backend.h:30-111, src/wav2vec2.cpp:104-125) and is
// written from ggml's published interface, not from ggml's source.
//
// The arithmetic behind ggml_mul_mat lives in ggml_shim.cpp and restates
// ggml's published CPU algorithm for quantized matmul (activations re-quantized
// to the weight's "vec_dot" type, block dot products accumulated in fp32).
#pragma once

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

// Type ids equal the GGUF tensor type ids (reference src/gguf.h:33-42).
enum ggml_type {
    GGML_TYPE_F32  = 0,
    GGML_TYPE_F16  = 1,
    GGML_TYPE_Q4_0 = 2,
    GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6,
    GGML_TYPE_Q5_1 = 7,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_Q8_1 = 9,
};

enum ggml_op {
    GGML_OP_NONE    = 0,
    GGML_OP_MUL_MAT = 1,
};

#define GGML_MAX_DIMS 4

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[GGML_MAX_DIMS];   // elements per dim, innermost first
    size_t  nb[GGML_MAX_DIMS];   // bytes per dim step
    enum ggml_op op;
    struct ggml_tensor * src[2];
    void * data;
};

struct ggml_context;
struct ggml_cgraph;

struct ggml_init_params {
    size_t mem_size;
    void * mem_buffer;
    bool   no_alloc;
};

struct ggml_context * ggml_init(struct ggml_init_params params);
void                  ggml_free(struct ggml_context * ctx);

size_t ggml_tensor_overhead(void);
size_t ggml_graph_overhead(void);
size_t ggml_nbytes(const struct ggml_tensor * t);

struct ggml_tensor * ggml_new_tensor_2d(struct ggml_context * ctx, enum ggml_type type,
                                        int64_t ne0, int64_t ne1);

// result[ne0 = a->ne[1], ne1 = b->ne[1]]: result[m][n] = dot(a row n, b row m)
struct ggml_tensor * ggml_mul_mat(struct ggml_context * ctx,
                                  struct ggml_tensor * a, struct ggml_tensor * b);

struct ggml_cgraph * ggml_new_graph(struct ggml_context * ctx);
void ggml_build_forward_expand(struct ggml_cgraph * gf, struct ggml_tensor * t);

#ifdef __cplusplus
}
#endif
