"""i_whisper_b200 -- B200-native (sm_100a) integer Whisper hot path.

Drop-in replacement for the CPU integer operators of vcsd-lab/I-Whisper
(``i_whisper.kernels._C``) and for the integer encoder + greedy decoder
forward of ``Whisper_int``, built on hand-written CUDA kernels behind the C
ABI in ``include/iwhisper_b200.h``.

Submodules:
  ops         -- ``<op>_cuda`` torch functions with the reference ``_C`` semantics
  model       -- ``WhisperIntB200``: GPU-resident encoder + greedy decoder (the
                 reference logit filters and argmax run on the device)
  checkpoint  -- ``i-whisper-int`` v1 checkpoint contract and seeded synthetic checkpoints
  frontend    -- log-mel + INT8 input quantisation on the GPU
  synthetic   -- seeded sine + noise audio windows
  sharding    -- utterance sharding across ranks
  microbench  -- kernel microbenchmarks through the C ABI
  build       -- in-tree nvcc build of ``_lib/libiwhisper_b200.so``
"""
__version__ = "0.1.0"
