// Single translation unit of libh3vae_b200.so: the device error word and all
// kernels live in one module, so no relocatable device code is needed.
#include "host_common.cu"
#include "mma_tc.cu"
#include "encoder_producers.cu"
#include "decoder_producers.cu"
#include "attention_tc.cu"
#include "conv_in.cu"
#include "conv_rgb.cu"
