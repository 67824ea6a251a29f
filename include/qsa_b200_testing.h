/*
 * qsa_b200_testing.h -- test hook of libqsa_b200.so. Not part of the decode
 * interface (include/qsa_b200.h): it exists so that a test can make the
 * tensor-core kernel's bounded waits run out on purpose, without a GPU fault,
 * and check that the failure reaches the host. No counterpart in the
 * reference (its kernels have no waits and no error path).
 */
#ifndef QSA_B200_TESTING_H_
#define QSA_B200_TESTING_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define QSA_B200_TESTING_API __attribute__((visibility("default")))
#else
#define QSA_B200_TESTING_API
#endif

/* Sets the limit, in nanoseconds, of every pipeline wait of the tensor-core
 * decode kernel launched from now on in this process (0 restores the
 * default of 1 s); returns the previous limit. A CTA whose wait runs out
 * records code 1 in the device error word (qsa_b200_device_error), waits
 * (with the 1 s limit) for its own copies and MMAs in flight, frees its
 * tensor memory and returns; its outputs are then undefined. Process-wide;
 * meant for tests only. */
QSA_B200_TESTING_API uint64_t qsa_b200_testing_set_wait_limit_ns(uint64_t ns);

#ifdef __cplusplus
}
#endif

#endif /* QSA_B200_TESTING_H_ */
