"""se12_b200: B200-native (sm_100a) SE12 lossless weight streaming.

SE12 stores BF16 weights losslessly in about 12 bits each; the kernels of
libse12_b200.so rebuild the exact BF16 values in registers inside a fused
GEMV. The package keeps the interface of the reference implementation
(Acaua-Rangel/se12, package ``lws``): the packed safetensors format, the
domain codec (``se12_b200.codec``), the GEMV entry point
(``se12_b200.gemv``), the GPU decoder (``se12_b200.decoder``) and the
runtime Linear replacement (``se12_b200.runtime``).
"""

__version__ = "0.1.0"
