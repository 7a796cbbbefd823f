/*
 * crexp.h -- TEST INFRASTRUCTURE ONLY.  Force-included (gcc -include) into
 * the diagnostic build of the reference, _ref/libmia_ref_crexp.so: after
 * <math.h> has been read, expf is renamed to oracle_expf_cr.  That build
 * differs from the stock one only in expf: the reference's two
 * calls (src/model/forward.c:99 softmax, :190 SiLU) get the correctly
 * rounded float of the double exp, the value the GPU computes, instead of
 * glibc's expf, which misrounds a few inputs in a million.  Comparing against
 * both builds separates an arithmetic difference of the GPU path (it would
 * show against both) from glibc's expf (it shows against the stock one only).
 */
#ifndef ORACLE_CREXP_H
#define ORACLE_CREXP_H
#include <math.h>
float oracle_expf_cr(float x);
#define expf oracle_expf_cr
#endif
