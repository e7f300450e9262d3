/* ORACLE -- test infrastructure only (see interp.c). */
#ifndef TCO_INTERP_H
#define TCO_INTERP_H
#include <stdint.h>

#define TCO_MAX_RANK 8

enum {
  TCO_INPUT = 0, TCO_CONST = 1,
  TCO_ADD = 2, TCO_SUB = 3, TCO_MUL = 4, TCO_DIV = 5,
  TCO_NEG = 6, TCO_EXP = 7, TCO_LOG = 8, TCO_RELU = 9, TCO_TANH = 10, TCO_STEP = 11, TCO_STOPGRAD = 12, TCO_SQRT = 13,
  TCO_MATMUL = 14, TCO_SUM = 15, TCO_MAX = 16,
  TCO_BROADCAST = 17, TCO_RESHAPE = 18, TCO_TRANSPOSE = 19
};

typedef struct tco_node {
  int32_t op, n_in, in0, in1;
  int32_t rank, axis, keep_dims, pad;
  int64_t shape[TCO_MAX_RANK];
  int32_t perm[TCO_MAX_RANK];
  const double* data;        /* input: its values; const: its values, or NULL for `scalar` */
  double scalar;             /* const value when data == NULL */
  const double* data_bound;  /* input, bounds mode: a carried bound (value used unrounded), or NULL */
  double* out;               /* if set, the node's value is written here */
  double* out_bound;         /* if set (bounds mode), the node's bound is written here */
} tco_node;

/* Evaluate every node in order; returns 0, or -1 with a message in err. */
int tco_evaluate(tco_node* nodes, int n, int with_bounds, char* err, int errlen);
int tco_abi_version(void);

#endif
