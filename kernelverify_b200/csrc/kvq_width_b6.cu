// Kernels for 6-bit codes.
#define KVQ_BITS 6
#include "kvq_width.inc"
