// Status codes returned by the C-ABI and error bits written by the kernels into the workspace.
#pragma once

#define SKINNY_OK 0
#define SKINNY_ERR_INVALID_ARG -1     /* null pointer or negative size */
#define SKINNY_ERR_SHAPE -2           /* K not a multiple of 64, N < 1, ... */
#define SKINNY_ERR_TOKENS -3          /* M outside [1, 16] */
#define SKINNY_ERR_ALIGNMENT -4       /* pointer or leading dimension not 16-byte aligned */
#define SKINNY_ERR_WORKSPACE -5       /* workspace missing or too small */
#define SKINNY_ERR_CUDA -6            /* a CUDA runtime call failed (see skinny_last_cuda_error) */
#define SKINNY_ERR_DEVICE -7          /* a kernel recorded an error bit in the workspace */
#define SKINNY_ERR_UNSUPPORTED -8     /* device is not sm_100 or option not supported */
#define SKINNY_ERR_SCRATCH_LIMIT -9   /* shape larger than the no-alloc entry's static scratch */

namespace skinny {
// Bits OR-ed into workspace word 0 by the kernels.  The wait bits mean a bounded wait on an
// mbarrier ran out (1 s); the kernel then stopped, released its tensor memory and returned.
constexpr unsigned kErrBitWaitFull = 1u << 0;
constexpr unsigned kErrBitWaitEmpty = 1u << 1;
constexpr unsigned kErrBitWaitAFull = 1u << 2;
constexpr unsigned kErrBitWaitAEmpty = 1u << 3;
constexpr unsigned kErrBitWaitDFull = 1u << 4;
constexpr unsigned kErrBitWaitDEmpty = 1u << 5;
constexpr unsigned kErrBitWaitDrain = 1u << 6;
constexpr unsigned kErrBitBadInput = 1u << 9;   // e.g. a token id outside the vocabulary
constexpr unsigned kErrBitWaitCluster = 1u << 10;  // a CTA's wait for its cluster peers' data
constexpr unsigned kErrBitWaitPeer = 1u << 11;     // a launch's wait for the other ranks' flags
}  // namespace skinny
