// The wide variant of the persistent decode step (head_dim of any 16-byte
// piece count, partially staged q rows, expert rows read from global memory,
// expert hidden sizes beyond one register segment): the kernels and phases of
// step.cu instantiated with kWide = true in a translation unit of their own,
// so that their out-of-line device functions do not share register
// allocation with the narrow variant's.
#define MIE_STEP_WIDE_TU 1
#include "step.cu"
