// The single translation unit of libtq4: device symbols (the status word) are shared between the
// parts without relocatable device code.
#include "weight.cu"
#include "gemv.cu"
#include "gemm.cu"
#include "api.cu"
#include "sharded.cu"
#include "noalloc.cu"
