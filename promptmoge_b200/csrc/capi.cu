// Library-level C ABI: version, status strings, device check, last CUDA error.
#include "common.cuh"

namespace pmg {
static thread_local int g_last_cuda_error = 0;
void set_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }
}  // namespace pmg

extern "C" int pmg_abi_version(void) { return 1; }

extern "C" const char* pmg_status_string(int status) {
    switch (status) {
        case PMG_OK: return "ok";
        case PMG_ERR_BAD_ARG: return "bad argument";
        case PMG_ERR_CUDA: return "CUDA runtime error";
        case PMG_ERR_TABLE_FULL: return "hash table full";
        case PMG_ERR_OVERFLOW: return "level capacity overflow";
        case PMG_ERR_UNSUPPORTED: return "unsupported configuration";
        case PMG_ERR_RANGE: return "coordinate outside the key range";
        case PMG_ERR_NO_DEVICE: return "no sm_100 device";
        case PMG_ERR_TIMEOUT: return "bounded wait expired inside a kernel";
        default: return "unknown status";
    }
}

extern "C" int pmg_last_cuda_error(void) { return pmg::g_last_cuda_error; }

extern "C" int pmg_check_device(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return PMG_ERR_NO_DEVICE;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) return PMG_ERR_NO_DEVICE;
    return (p.major == 10 && p.minor == 0) ? PMG_OK : PMG_ERR_NO_DEVICE;
}
