// sf_fused_encode_noalloc: the fused encoder for callers that cannot allocate device memory.
//
// sf_fused_encode needs a workspace (the b_dec-shifted copy of x) that its caller
// allocates. Some callers cannot: a foreign-language host (Go, Java, Node through the C
// ABI) that is handed only the input and output buffers by the framework owning the GPU;
// a process whose caching allocator has already reserved nearly all device memory, so a
// fresh cudaMalloc fails; or a latency-bound loop that cannot afford cudaMalloc's
// implicit device synchronisation. This entry point takes its workspace from a
// fixed-size array in the library's device image instead, and allocates nothing.
#include <mutex>

#include "sf_common.cuh"
#include "sf_internal.h"

namespace {

// 16 MiB of device scratch. Every GPU on which the library's device code is loaded
// holds this array until the process exits.
constexpr size_t kScratchBytes = 16u << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void *g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device. In host code the array's
// name is only a host-side stand-in, so the address is looked up once per device, with
// that device current, and cached for the life of the process. cudaDeviceReset unloads
// the library's device image and may move the array, so calls after a reset of that
// device are unsupported.
int scratch_address(void **out) {
    int dev = -1;
    int st = sf::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (st) return st;
    if (dev < 0 || dev >= kMaxDevices) return sf::set_error(SF_ERR_UNSUPPORTED, "device ordinal %d too large", dev);
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        st = sf::check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
        if (st) return st;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return SF_OK;
}

}  // namespace

extern "C" {

SF_API int sf_fused_encode_noalloc(const sf_matrix *x, const sf_matrix *W_enc, const sf_vector *b_enc,
                                   const sf_vector *b_dec, const sf_vector *threshold, int activation,
                                   const sf_matrix *out, int32_t *row_nnz, int allow_tf32, int variant,
                                   sf_stream stream) {
    // IEEE fp32 products (fp32 x and W_enc, TF32 not allowed) run split-precision on the
    // tensor cores by default, and the split copy of W_enc (three bf16 parts) outgrows the
    // static scratch for any real SAE: here the CUDA-core IEEE kernel, which needs only the
    // shifted x, serves those calls.
    const bool ieee = x && W_enc && x->dtype == SF_F32 && W_enc->dtype == SF_F32 && !allow_tf32;
    if (ieee && variant == SF_VARIANT_AUTO) variant = SF_VARIANT_SIMT;
    size_t need = 0;
    int st = sf_fused_encode_workspace(x, W_enc, allow_tf32, variant, &need);
    if (st) return st;
    if (need > kScratchBytes) {
        // The workspace of a zero-row x is the repacked copy of W_enc alone: nonzero when the
        // tensor-core kernel cannot read W_enc in place. Fewer rows cannot shrink that part.
        sf_matrix x0 = *x;
        x0.rows = 0;
        size_t w_part = 0;
        st = sf_fused_encode_workspace(&x0, W_enc, allow_tf32, variant, &w_part);
        if (st) return st;
        if (w_part + 256 > kScratchBytes && ieee)
            return sf::set_error(SF_ERR_WORKSPACE,
                                 "sf_fused_encode_noalloc: IEEE fp32 on the tensor cores needs a split copy of "
                                 "W_enc (%zu bytes) that does not fit the %zu-byte static scratch. Pass variant "
                                 "SF_VARIANT_AUTO or SF_VARIANT_SIMT (the CUDA-core IEEE kernel), or call "
                                 "sf_fused_encode with a workspace.",
                                 w_part, kScratchBytes);
        if (w_part + 256 > kScratchBytes)
            return sf::set_error(SF_ERR_WORKSPACE,
                                 "sf_fused_encode_noalloc: W_enc is in a layout the tensor-core kernel cannot read "
                                 "in place, and its repacked copy (%zu bytes) does not fit the %zu-byte static "
                                 "scratch. Pass a 16-bit W_enc contiguous along one dimension with a 16-byte-aligned "
                                 "base and row pitch, or an fp32 W_enc in column-major layout for TF32, or call "
                                 "sf_fused_encode with a workspace.",
                                 w_part, kScratchBytes);
        return sf::set_error(SF_ERR_WORKSPACE,
                             "sf_fused_encode_noalloc needs %zu bytes of scratch for these operands; its static "
                             "scratch holds %zu bytes. Call it on fewer rows of x at a time.",
                             need, kScratchBytes);
    }
    void *scratch = nullptr;
    st = scratch_address(&scratch);
    if (st) return st;
    // The shifted copy of x (and a repacked W_enc, if any) is written in full before the
    // GEMM reads it, so nothing in the shared scratch has to start at zero.
    return sf_fused_encode(x, W_enc, b_enc, b_dec, threshold, activation, out, row_nnz, allow_tf32, variant,
                           scratch, kScratchBytes, stream);
}

}  // extern "C"
