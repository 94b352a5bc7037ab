// fhessm.cu -- single translation unit of libfhessm.so (the kernels share one
// __constant__ table of moduli, so the sources are compiled together).
#include "kernels.cu"
#include "ntt.cu"
#include "engine.cu"
#include "ksbatch.cu"
#include "circuit.cu"
#include "matvec.cu"
#include "bootstrap.cu"
#include "model.cu"
#include "capi.cu"
#include "serve.cu"
#include "noalloc.cu"
