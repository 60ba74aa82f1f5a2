// noalloc.cu — the greedy head (out_norm, text_linear, argmax) for callers that cannot
// allocate device memory.
//
// The head's argmax needs scratch: every CTA of the logits product leaves its best
// (value, index) per stream in global memory and the last CTA to finish, elected by a
// counter, reduces them. svl_stt_step keeps that scratch in the state it allocated.
// Callers that own the allocation policy of the process -- a host whose memory pool hands
// out no device memory of its own to plugins, code running where cudaMalloc would
// synchronise the device mid-stream, or a real-time audio thread that must never enter the
// allocator -- cannot create states. For them this file keeps the scratch in a fixed
// static __device__ array, which every GPU that loads the library holds until the process
// exits.
#include <mutex>

#include "engine.h"

using svl::Error;

namespace {

// Scratch of one head launch: the counter that elects the last CTA (padded to 256 bytes),
// then the per-CTA candidates, values then indices, for up to kNoAllocMaxBatch streams.
constexpr int kNoAllocMaxBatch = svl::kMaxNbChunk;  // 8 streams per call
constexpr size_t kCandidates = (size_t)kNoAllocMaxBatch * svl::kLogitsGrid;
constexpr size_t kScratchBytes = 256 + kCandidates * 4 * 2;  // 19,200 bytes

static __device__ __align__(256) unsigned char g_head_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
unsigned char* g_scratch_ptr[kMaxDevices];

// The device address of the scratch on `device` (the current device). In host code the
// array's name is only a host-side stand-in, so the address comes from the runtime. It is
// stored once the lookup succeeds; a failed lookup (for instance one made inside a stream
// capture) is reported and tried again on the next call.
unsigned char* scratch_on(int device) {
  if (device < 0 || device >= kMaxDevices) throw Error(SVL_ERR_CUDA, "device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_head_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      throw Error(SVL_ERR_CUDA, std::string("cudaGetSymbolAddress of the head scratch: ") +
                                    cudaGetErrorString(e));
    }
    g_scratch_ptr[device] = static_cast<unsigned char*>(p);
  }
  return g_scratch_ptr[device];
}

}  // namespace

extern "C" SVL_API svl_status svl_stt_head_noalloc(svl_model* model, int32_t batch,
                                                   const float* d_hidden, uint32_t* d_tokens,
                                                   float* d_logits, void* cuda_stream) {
  try {
    if (!model || !d_hidden || !d_tokens) throw Error(SVL_ERR_INVALID_INPUT, "null argument");
    svl::Model& m = *model->m;
    if (m.kind != 0) throw Error(SVL_ERR_INVALID_INPUT, "not an STT model");
    if (batch < 1 || batch > kNoAllocMaxBatch)
      throw Error(SVL_ERR_INVALID_INPUT,
                  "svl_stt_head_noalloc: batch must be 1..8 (its fixed scratch holds the "
                  "argmax candidates of 8 streams); call it once per group of 8 streams");
    svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
    unsigned char* scratch = scratch_on(m.device);
    cudaStream_t st = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : m.stream;
    // The counter must start at zero; the candidates are all written before they are read.
    svl::check_cuda(cudaMemsetAsync(scratch, 0, sizeof(unsigned), st), "clear head scratch");
    svl::GemvParams g{};
    const svl::Linear& L = m.text_linear;
    g.w = L.w.as<uint8_t>();
    g.row_stride = L.row_stride;
    g.n = L.n;
    g.k = L.k;
    g.wtype = L.wtype;
    g.x = d_hidden;
    g.x_stride = m.cfg.d_model;
    g.nb = batch;
    g.norm = m.out_norm.kind;
    g.norm_w = m.out_norm.w.as<float>();
    g.norm_b = m.out_norm.b.as<float>();
    g.eps = m.out_norm.eps;
    g.bias = L.bias.as<float>();
    g.epi = svl::EPI_LOGITS;
    g.out = d_logits;
    g.out_stride = L.n;
    g.am_ticket = reinterpret_cast<unsigned*>(scratch);
    g.am_val = reinterpret_cast<float*>(scratch + 256);
    g.am_idx = reinterpret_cast<int*>(scratch + 256 + kCandidates * 4);
    g.tokens = d_tokens;
    svl::launch_gemv(g, st);
    svl::check_cuda(cudaGetLastError(), "head launch");
    return SVL_OK;
  } catch (const Error& e) {
    svl::set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    svl::set_last_error(e.what());
    return SVL_ERR_CUDA;
  }
}
