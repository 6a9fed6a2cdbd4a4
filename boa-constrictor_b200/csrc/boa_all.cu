// boa_all.cu -- the library's single translation unit.  Kernels, launchers and
// the host runtime are compiled together so that device globals (the error
// word read back by the host) have exactly one definition without relocatable
// device code.
#include "gemm.cu"
#include "mlp.cu"
#include "mamba.cu"
#include "rnn.cu"
#include "runtime.cpp"
#include "container.cpp"
#include "noalloc.cu"
#include "coder_api.cu"
#include "pyrc.cu"
