"""marian_cuda: B200 backend for marian-edge's Q8 greedy translation path.

The compute path is ``libmarian_cuda.so`` (CUDA kernels for sm_100a behind a
C ABI declared in ``include/marian_cuda.h``).  This package is the host-side
mirror of marian-edge's backend interface over that ABI:

* :mod:`marian_cuda.backend` -- ``CudaEngine`` (the ``CpuTokenEngine`` seam,
  ``translate_token_ids``) and ``CudaBackend`` (``TranslationBackend``);
* :mod:`marian_cuda.marian_bin` -- Marian binary v1 writer/reader;
* :mod:`marian_cuda.workloads` -- seeded synthetic models and request streams.
"""
