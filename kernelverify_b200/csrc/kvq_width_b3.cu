// Kernels for 3-bit codes.
#define KVQ_BITS 3
#include "kvq_width.inc"
