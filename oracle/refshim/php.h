/*
 * Minimal stand-in for the PHP header, so that the reference's
 * src/data_types.c compiles on its own for oracle/_ref.  data_types.c uses
 * Zend only in dtype_from_zval(), which no test calls; these definitions
 * exist to satisfy the compiler, not to emulate Zend.
 */
#ifndef PT_REFSHIM_PHP_H
#define PT_REFSHIM_PHP_H
#include <stdint.h>
typedef struct pt_refshim_zval { int type; union { long long l; double d; } v; } zval;
#define IS_FALSE 2
#define IS_TRUE 3
#define IS_LONG 4
#define IS_DOUBLE 5
#define Z_TYPE_P(z) ((z)->type)
#define Z_LVAL_P(z) ((z)->v.l)
#define Z_DVAL_P(z) ((z)->v.d)
#endif
