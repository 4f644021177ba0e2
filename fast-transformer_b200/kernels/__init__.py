"""B200 (sm_100a) CUDA kernels behind the reference engine's kernel-wrapper API.

Module and function names mirror john-jpet/fast-transformer's ``engine/kernels``
package, so the engine's call sites (engine/layers.py, engine/decode.py) bind to these
without change. Every function launches hand-written CUDA from libfastb200.so on the
current stream; none has a CPU or Triton path.
"""
