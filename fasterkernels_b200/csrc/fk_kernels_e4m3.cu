// fk_kernels_e4m3.cu -- the decode kernel instantiations for E4M3 KV
// (compiled apart from the host side so that the kernel sets build in
// parallel; see fk_decode_kernel.cuh).
#include "fk_decode_kernel.cuh"

FK_KERNELS_E4M3(FK_KERNEL_INST)
