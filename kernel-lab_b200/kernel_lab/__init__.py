"""kernel-lab's two memory-bound inference hot paths, rebuilt for B200 (sm_100a).

Drop-in for kernel-lab's ``kernel_lab`` package on the CUDA path: ``kernel_lab.cuda_ops``
keeps its API and ``import kernel_lab._C`` registers the same ``torch.ops.kernel_lab``
schemas. The kernels live in ``libkernel_lab_b200.so`` behind a C ABI
(``include/kernel_lab_b200.h``); ``kernel_lab.capi`` binds it with ctypes.
"""

__version__ = "0.1.0"
