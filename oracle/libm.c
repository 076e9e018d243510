/*
 * libm.c — the transcendental functions of the oracle.
 * TEST INFRASTRUCTURE ONLY (see sg_oracle.h).
 *
 * The reference calls f32::exp / sin / cos (smollm_chat.rs:586-588,
 * :1200-1203, :1397-1420, :3463-3495), which Rust's std takes from the
 * platform libm: glibc's expf, sinf and cosf on Linux.  The oracle calls the
 * same functions of the host's glibc.  (The CUDA kernels compute glibc's
 * results bit for bit from a restatement of its algorithm; tests/test_libm.py
 * checks that restatement against this same libm over every float.)
 */
#include <math.h>

#include "sg_oracle.h"

float or_expf(float x) { return expf(x); }
float or_sinf(float x) { return sinf(x); }
float or_cosf(float x) { return cosf(x); }
