"""i_whisper_b200 -- B200-native (sm_100a) integer Whisper hot path.

Drop-in replacement for the CPU integer operators of vcsd-lab/I-Whisper
(``i_whisper.kernels._C``) and for the integer encoder + greedy decoder
forward of ``Whisper_int``, built on hand-written CUDA kernels behind the C
ABI in ``include/iwhisper_b200.h``.

Submodules:
  ops       -- ``<op>_cuda`` torch functions with the reference ``_C`` semantics
  model     -- ``WhisperIntB200``: GPU-resident encoder + greedy decoder
  decoding  -- greedy loop with the reference logit filters
  build     -- in-tree nvcc build of ``_lib/libiwhisper_b200.so``
"""
__version__ = "0.1.0"
