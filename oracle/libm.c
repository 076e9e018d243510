/*
 * libm.c — the transcendental functions of the oracle.
 * TEST INFRASTRUCTURE ONLY (see sg_oracle.h).
 *
 * The reference calls f32::exp / sin / cos, which Rust's std takes from the
 * platform libm (glibc expf, sinf, cosf on Linux, within about half an ulp but
 * not correctly rounded).  The CUDA kernels compute the correctly rounded value
 * instead (the double-precision function rounded to float).  Mode 0 (default)
 * is glibc, mode 1 the correctly rounded value: with mode 1 the oracle and the
 * GPU share every rounding, so a test can check the rest of the arithmetic bit
 * for bit, and a second test measures what the libm choice alone changes.
 */
#include <math.h>

#include "sg_oracle.h"

static int cr_math;

void or_set_cr_math(int on) { cr_math = on != 0; }
int or_cr_math(void) { return cr_math; }

float or_expf(float x) { return cr_math ? (float)exp((double)x) : expf(x); }
float or_sinf(float x) { return cr_math ? (float)sin((double)x) : sinf(x); }
float or_cosf(float x) { return cr_math ? (float)cos((double)x) : cosf(x); }
