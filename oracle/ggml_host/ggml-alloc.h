/*
 * ggml-alloc.h -- TEST INFRASTRUCTURE ONLY: host-only stand-in for the ggml
 * graph-allocator names the reference's decoder sources use (see ggml.h in
 * this directory). None of these is reached on the decoder's CPU branch.
 */
#pragma once

#include "ggml-backend.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ggml_gallocr * ggml_gallocr_t;

ggml_gallocr_t        ggml_gallocr_new(ggml_backend_buffer_type_t buft);
void                  ggml_gallocr_free(ggml_gallocr_t galloc);
bool                  ggml_gallocr_alloc_graph(ggml_gallocr_t galloc, struct ggml_cgraph * graph);
ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(struct ggml_context * ctx, ggml_backend_t backend);

#ifdef __cplusplus
}
#endif
