"""cuda_tempiler_b200: the sm_100a (B200) GEMM backend and ``tempo/arch/1`` plugin of the
tempolator.  The compute path is ``libtempo_sm100.so`` (hand-written tcgen05/TMA kernels,
C-ABI in include/tempo_sm100.h); torch supplies device memory, streams and NCCL plumbing."""

__version__ = "0.1.0"
