// fk_kernels_bf16.cu -- the decode kernel instantiations for BF16 KV
// (compiled apart from the host side so that the kernel sets build in
// parallel; see fk_decode_kernel.cuh).
#include "fk_decode_kernel.cuh"

FK_KERNELS_BF16(FK_KERNEL_INST)
