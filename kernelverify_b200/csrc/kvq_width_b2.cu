// Kernels for 2-bit codes.
#define KVQ_BITS 2
#include "kvq_width.inc"
