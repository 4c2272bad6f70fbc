// fz_status.h -- error reporting shared by the C ABI translation units of libzf_featurize.so (defined in fz_capi.cu):
// a failed call records "ZipNeRF: <message>" for the calling thread's zf_last_error() and returns its status code.
#pragma once

#include <cuda_runtime.h>

#include <string>

namespace zf {

int set_error(int code, const std::string& message);
int set_cuda_error(cudaError_t error, const char* what);

}  // namespace zf
