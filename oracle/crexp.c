/* crexp.c -- TEST INFRASTRUCTURE ONLY (see crexp.h): expf as the float
 * nearest the double exp, for the diagnostic build of the reference. */
#include <math.h>

#include "crexp.h"

float oracle_expf_cr(float x) { return (float)exp((double)x); }
