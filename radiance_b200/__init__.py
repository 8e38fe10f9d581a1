"""radiance_b200: a B200-native (sm_100a) NVFP4 linear-layer path for the radiance training
framework.  ``radiance_b200.nvfp4`` is the drop-in for ``radiance.nvfp4``; the kernels live in
``radiance_b200/csrc`` behind the C ABI of ``include/radiance_nvfp4.h``."""

__version__ = "0.1.0"
