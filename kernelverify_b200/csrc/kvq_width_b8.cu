// Kernels for 8-bit codes.
#define KVQ_BITS 8
#include "kvq_width.inc"
