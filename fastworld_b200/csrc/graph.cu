// Library-held CUDA graphs and peer access for checkpoint placement.
//
// fastworld records each chunk variant (first / steady x generate / prefill) as a CUDA graph
// through torch (fastworld/graph.py:13-33).  Here the engine's launch calls are recorded by
// stream capture into executable graphs that the library owns: one launch of the recorded
// chunk replays every kernel with its parameters and buffer pointers baked in, on any stream.
// Recording executes nothing, so it neither reads nor writes the session state.
#include <cuda_runtime.h>

#include "../../include/fastworld_b200.h"

struct fw_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

extern "C" {

int fw_graph_begin(void* stream) {
  if (!stream) return FW_EINVAL;   // the legacy default stream cannot be captured
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &st) != cudaSuccess) return FW_ECUDA;
  if (st != cudaStreamCaptureStatusNone) return FW_ESTATE;
  return cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess ? FW_OK : FW_ECUDA;
}

int fw_graph_end(void* stream, fw_graph** out) {
  if (!stream || !out) return FW_EINVAL;
  *out = nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaGraph_t g = nullptr;
  // Ending the capture is required even when recording failed, or the stream stays unusable.
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (e != cudaSuccess || !g) {
    if (g) cudaGraphDestroy(g);
    return FW_ECUDA;
  }
  cudaGraphExec_t x = nullptr;
  if (cudaGraphInstantiateWithFlags(&x, g, 0) != cudaSuccess) {
    cudaGraphDestroy(g);
    return FW_ECUDA;
  }
  fw_graph* h = new fw_graph;
  h->graph = g;
  h->exec = x;
  *out = h;
  return FW_OK;
}

int fw_graph_launch(const fw_graph* g, void* stream) {
  if (!g || !g->exec) return FW_EINVAL;
  return cudaGraphLaunch(g->exec, static_cast<cudaStream_t>(stream)) == cudaSuccess ? FW_OK : FW_ECUDA;
}

int fw_graph_nodes(const fw_graph* g, size_t* n) {
  if (!g || !n) return FW_EINVAL;
  *n = 0;
  return cudaGraphGetNodes(g->graph, nullptr, n) == cudaSuccess ? FW_OK : FW_ECUDA;
}

void fw_graph_destroy(fw_graph* g) {
  if (!g) return;
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  delete g;
}

int fw_peer_access(int peer) {
  int dev = 0, n = 0, ok = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceCount(&n) != cudaSuccess) return FW_ECUDA;
  if (peer < 0 || peer >= n) return FW_EINVAL;
  if (peer == dev) return FW_OK;
  if (cudaDeviceCanAccessPeer(&ok, dev, peer) != cudaSuccess) return FW_ECUDA;
  if (!ok) return FW_EINVAL;
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();   // clear the (non-sticky) "already enabled" error
    return FW_OK;
  }
  return e == cudaSuccess ? FW_OK : FW_ECUDA;
}

}  // extern "C"
