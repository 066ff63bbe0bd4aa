// cuda13_compat.h -- force-included when the reference backend is compiled for
// the parity harness with CUDA 12.9.  The reference's host-side graph code
// (its nerf_configure_training, used by the harness only to time the
// reference's own training step) uses four CUDA 13 runtime entry points; this
// header maps them onto their 12.9 equivalents.  Device code is untouched.
#pragma once
#include <cuda_runtime.h>

typedef void* cudaExecutionContext_t;

// CUDA 13 names the execution context a conditional node's body runs in; with
// 12.9 the body always runs in the graph's own context, so any non-null token
// lets the reference's graph set-up proceed (the one line that stores it in
// the node parameters is disabled by the Makefile's patch).
static inline cudaError_t cudaDeviceGetExecutionCtx(cudaExecutionContext_t* ctx, int) {
    static int token;
    *ctx = &token;
    return cudaSuccess;
}

static inline cudaError_t cudaGraphConditionalHandleCreate_v2(cudaGraphConditionalHandle* handle, cudaGraph_t graph,
                                                              cudaExecutionContext_t, unsigned int default_value,
                                                              unsigned int flags) {
    return cudaGraphConditionalHandleCreate(handle, graph, default_value, flags);
}

// CUDA 13 signature (7 arguments) on the 12.9 _v3 entry point.
static inline cudaError_t nerf_ref_stream_capture_info(cudaStream_t s, cudaStreamCaptureStatus* status,
                                                       unsigned long long* id, cudaGraph_t* graph,
                                                       const cudaGraphNode_t** deps, const cudaGraphEdgeData** edges,
                                                       size_t* n) {
    return cudaStreamGetCaptureInfo_v3(s, status, id, graph, deps, edges, n);
}
#undef cudaStreamGetCaptureInfo
#define cudaStreamGetCaptureInfo nerf_ref_stream_capture_info

// CUDA 13 signature (6 arguments, with edge data) on the 12.9 _v2 entry point.
static inline cudaError_t nerf_ref_graph_add_node(cudaGraphNode_t* node, cudaGraph_t graph, const cudaGraphNode_t* deps,
                                                  const cudaGraphEdgeData* edges, size_t n, cudaGraphNodeParams* params) {
    return cudaGraphAddNode_v2(node, graph, deps, edges, n, params);
}
#define cudaGraphAddNode nerf_ref_graph_add_node
