// Kernels for 4-bit codes.
#define KVQ_BITS 4
#include "kvq_width.inc"
