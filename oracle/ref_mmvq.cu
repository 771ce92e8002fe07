// ref_mmvq.cu — the reference's own GPU Q4_K matvec (vendored ggml-cuda
// mul_mat_vec_q<GGML_TYPE_Q4_K> with its quantize_q8_1 activation
// quantizer, ggml-cuda/mmvq.cu:393 and quantize.cu:5), compiled for sm_100a
// from the reference tree by oracle/Makefile into oracle/_ref/libmmvq_ref.so.
// TEST INFRASTRUCTURE AND GPU COMPARISON POINT ONLY: nothing of the product
// links it. The reference sources are included where they lie; this file
// adds only the four CUDA-backend symbols they call (device info, error
// report, get / set device), answered from the CUDA runtime, and one C
// entry point that runs the same two launches ggml_cuda_mul_mat_vec_q makes
// (mmvq.cu:1029-1110) for a plain 2-D weight and B activation columns.
#include "mmvq.cu"
#include "quantize.cu"

#include <cstdio>
#include <cstdlib>

static ggml_cuda_device_info g_info;
static bool g_info_ready = false;

const ggml_cuda_device_info& ggml_cuda_info() {
    if (!g_info_ready) {
        int n = 0;
        cudaGetDeviceCount(&n);
        g_info.device_count = n < GGML_CUDA_MAX_DEVICES ? n : GGML_CUDA_MAX_DEVICES;
        for (int d = 0; d < g_info.device_count; ++d) {
            cudaDeviceProp p;
            cudaGetDeviceProperties(&p, d);
            g_info.devices[d].cc = 100 * p.major + 10 * p.minor;
            g_info.devices[d].nsm = p.multiProcessorCount;
            g_info.devices[d].smpb = p.sharedMemPerBlock;
            g_info.devices[d].smpbo = p.sharedMemPerBlockOptin;
            g_info.devices[d].warp_size = p.warpSize;
            g_info.devices[d].total_vram = p.totalGlobalMem;
        }
        g_info_ready = true;
    }
    return g_info;
}

void ggml_cuda_error(const char* stmt, const char* func, const char* file, int line, const char* msg) {
    fprintf(stderr, "ggml-cuda error: %s in %s at %s:%d: %s\n", stmt, func, file, line, msg);
    abort();
}

void ggml_cuda_set_device(int device) { cudaSetDevice(device); }

int ggml_cuda_get_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

std::unique_ptr<ggml_cuda_pool> ggml_backend_cuda_context::new_pool_for_device(int, int) { abort(); }

// y [ncols_dst][nrows] = W [nrows rows of ncols Q4_K values] . x [ncols_dst][ncols]
// (fp32, device), quantized to Q8_1 into xq (ncols_dst * refmmvq_xq_bytes(ncols)
// bytes of device scratch) on the given stream.
extern "C" size_t refmmvq_xq_bytes(int ncols) {
    return (size_t)GGML_PAD(ncols, MATRIX_ROW_PADDING) / QK8_1 * sizeof(block_q8_1);
}

extern "C" int refmmvq_q4k(const void* w, int nrows, int ncols, const float* x, int ncols_dst, void* xq, float* y,
                           void* stream) {
    if (ncols % QK_K || ncols_dst < 1 || ncols_dst > MMVQ_MAX_BATCH_SIZE) return -1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t ne10_padded = GGML_PAD(ncols, MATRIX_ROW_PADDING);
    quantize_row_q8_1_cuda(x, nullptr, xq, GGML_TYPE_Q4_K, ncols, ncols, (int64_t)ncols * ncols_dst,
                           (int64_t)ncols * ncols_dst, ne10_padded, ncols_dst, 1, 1, s);
    ggml_cuda_mm_fusion_args_device fusion{};
    mul_mat_vec_q_switch_ncols_dst<GGML_TYPE_Q4_K>(w, xq, nullptr, fusion, y, ncols, nrows, ncols_dst, ncols / QK_K,
                                                   (int)(ne10_padded / QK8_1), nrows, 1, 1, 1, 0, 0, 0, 1, 1, 0, 0, 0,
                                                   0, s);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
