// Unity build of libltxb200.so: one translation unit, so the device error word and the
// shared device helpers need no relocatable device code.
#include "api.cu"
#include "philox.cu"
#include "elementwise.cu"
#include "gemm.cu"
#include "attention.cu"
#include "parallel.cu"
#include "vae.cu"
#include "dit_step.cu"
