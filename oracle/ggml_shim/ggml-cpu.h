// ggml CPU-compute entry point used by the reference (src/ggml_backend.h:106).
// Part of the oracle's ggml-API shim; see ggml.h for scope.
#pragma once
#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

// Computes every node of the graph with n_threads host threads.
// Returns 0 on success (ggml returns GGML_STATUS_SUCCESS == 0).
int ggml_graph_compute_with_ctx(struct ggml_context * ctx, struct ggml_cgraph * gf, int n_threads);

#ifdef __cplusplus
}
#endif
