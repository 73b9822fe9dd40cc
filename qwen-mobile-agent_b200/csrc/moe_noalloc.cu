// moe_noalloc.cu -- the MoE FFN block for callers that cannot allocate
// device memory.
//
// Who needs it: a host process that has reserved the device's memory for its
// own pools and lets no library allocate behind its back (a serving process
// with a fixed memory budget), or a caller whose step loop cannot afford the
// implicit device synchronisation and latency of cudaMalloc.  Such callers
// cannot provide the scratch buffer qma_cuda_moe_layer asks for, so this
// entry point keeps its scratch in a fixed array inside the library instead.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds it until the process exits.  Host code cannot use the
// array's name as a device address (in host code it names a host-side
// stand-in), so the device address is looked up with cudaGetSymbolAddress
// once per device, with that device current, the first time the entry point
// runs on it.  That first call on a device should therefore come before any
// stream capture on that device.
//
// Every call shares the one array.  Calls whose kernels overlap on the GPU
// (different streams, or different host threads, without ordering between
// them) race on it and must not be issued.  The array keeps whatever the
// previous call left; the parts that must start at zero (the completion
// counters) are cleared by every call before its kernels run, and all other
// parts are written before they are read within a call.
#include <mutex>

#include "common.cuh"
#include "moe.cuh"

namespace qma {

// Sized for QMA_CUDA_MOE_NOALLOC_MAX_T tokens (moe_scratch_bytes(4) is
// about 404 KB); checked against moe_scratch_bytes() at set-up.
constexpr size_t NOALLOC_SCRATCH_BYTES = 512 * 1024;
static __device__ __align__(256) uint8_t g_moe_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
static void *g_noalloc_ptr[NOALLOC_MAX_DEVICES];
static std::mutex g_noalloc_mu;

// Device address of this device's copy of the scratch array (set-up on
// first use: the current device is the one the call runs on).
static int noalloc_scratch(void **out) {
    int dev = -1;
    QMA_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) {
        set_error("qma_cuda_moe_layer_noalloc: device %d beyond the %d supported", dev,
                  NOALLOC_MAX_DEVICES);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            set_error("qma_cuda_moe_layer_noalloc: cudaGetSymbolAddress of the scratch array "
                      "failed on device %d: %s", dev, cudaGetErrorString(e));
            return QMA_CUDA_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return QMA_CUDA_OK;
}

}  // namespace qma

extern "C" int qma_cuda_moe_layer_noalloc(const qma_cuda_moe_weights *w, const float *x2, int T,
                                          float *x_out, int32_t *sel, float *wts,
                                          void *stream) {
    qma::clear_error();
    QMA_REQUIRE(w && x2 && x_out && T > 0, "qma_cuda_moe_layer_noalloc: bad arguments (T %d)", T);
    QMA_REQUIRE(qma::aligned_to(x2, 16) && qma::aligned_to(x_out, 16),
                "qma_cuda_moe_layer_noalloc: x2 / x_out must be 16-byte aligned");
    if (T > QMA_CUDA_MOE_NOALLOC_MAX_T) {
        qma::set_error("qma_cuda_moe_layer_noalloc: T = %d tokens exceeds the fixed scratch "
                       "capacity of %d tokens; use qma_cuda_moe_layer with caller scratch",
                       T, QMA_CUDA_MOE_NOALLOC_MAX_T);
        return QMA_CUDA_ERR_INVALID;
    }
    QMA_REQUIRE(w->post_norm && w->gate_inp && w->gate_exps && w->up_exps && w->down_exps &&
                    w->gate_inp_shexp && w->gate_shexp && w->up_shexp && w->down_shexp,
                "qma_cuda_moe_layer_noalloc: missing weight pointer");
    QMA_REQUIRE(w->down_type == QMA_TYPE_Q6_K || w->down_type == QMA_TYPE_Q4_K,
                "qma_cuda_moe_layer_noalloc: down_type %d must be Q6_K or Q4_K", w->down_type);
    QMA_REQUIRE(w->down_shexp_type == w->down_type,
                "qma_cuda_moe_layer_noalloc: shared and routed down projections must share a type");
    if (qma::moe_scratch_bytes(QMA_CUDA_MOE_NOALLOC_MAX_T) > qma::NOALLOC_SCRATCH_BYTES) {
        qma::set_error("qma_cuda_moe_layer_noalloc: built-in scratch too small");
        return QMA_CUDA_ERR_STATE;
    }
    void *scratch = nullptr;
    const int rc = qma::noalloc_scratch(&scratch);
    if (rc) return rc;
    return qma::moe_layer(*w, x2, T, x_out, sel, wts, scratch, qma::as_stream(stream), true);
}
