/* hx_oracle_lib.h -- TEST INFRASTRUCTURE ONLY: the oracle's library-mechanism
 * steps (hx_oracle_lib.c), called from the step sequence in hx_oracle.c. */
#ifndef HX_ORACLE_LIB_H
#define HX_ORACLE_LIB_H

#include "hx_oracle.h"

struct hxo_libstate;
int hxo_lib_alloc(const hxo_group* g, struct hxo_libstate** out);
void hxo_lib_free(struct hxo_libstate* L);
void hxo_lib_init(const hxo_group* g, struct hxo_libstate* L, const double* v);
void hxo_lib_current(const hxo_group* g, struct hxo_libstate* L, const double* v, double* rhs, double* d);
void hxo_lib_state_ion(const hxo_group* g, struct hxo_libstate* L, const double* v);
void hxo_lib_state(const hxo_group* g, struct hxo_libstate* L, const double* v);
int hxo_lib_final(const hxo_group* g, const struct hxo_libstate* L, double* out, int cap);

#endif
