// fz_inst.cu -- compiled once per instantiation object by the build (separate objects compile in parallel):
//   -DZF_INST_F=F -DZF_INST_PAD=0   the forward without MLP and the NeRF-level backward of F (F == 1: also the debug
//                                   kernel)
//   -DZF_INST_F=F -DZF_INST_PAD=P   the MLP forward and the proposal-level backward of (F, P)
#include "fz_kernel_set.h"

#if !defined(ZF_INST_F) || !defined(ZF_INST_PAD)
#error "compile with -DZF_INST_F=<features> -DZF_INST_PAD=<padded mlp inputs or 0>"
#endif

#if ZF_INST_PAD == 0
extern "C" const zf::KernelSet ZF_KSET_NAME(ZF_INST_F) = {
    zf::fz_forward_kernel<ZF_INST_F, 0>,
    zf::fz_backward_kernel<ZF_INST_F>,
};
#if ZF_INST_F == 1
extern "C" void (*const zf_debug_kernel)(zf::GridParams, zf::DebugArgs) = zf::fz_debug_kernel<0>;
extern "C" void (*const zf_check_erf_kernel)(uint32_t, uint32_t, unsigned long long*, uint32_t*) = zf::fz_check_erf_kernel<0>;
#endif
#else
extern "C" const zf::MlpKernelSet ZF_MLP_KSET_NAME(ZF_INST_F, ZF_INST_PAD) = {
    zf::fz_forward_kernel<ZF_INST_F, ZF_INST_PAD>,
    zf::fz_backward_mlp_kernel<ZF_INST_F, ZF_INST_PAD>,
};
#endif
