/*
 * run_graph.c -- a host with no language runtime of its own driving the whole path through libtcb200:
 * the graph (the reference's Graph.toJSON form) is lowered by tc_lower_json, run by tc_lowered_run, and
 * every node's float32 value is written out.  Test infrastructure: tests/test_gpu_lower_abi.py builds it
 * with gcc and compares its output with the Python host's, bit for bit.
 *
 *   run_graph GRAPH.json OPTS.json INPUTS.bin OUT.bin
 *
 * INPUTS.bin holds, for every input node in node order, its float32 values; OUT.bin receives every node's
 * values in node order (the sizes come from the lowering's record, so this program reads the node
 * shapes from GRAPH.json's "shape" arrays with a minimal scan).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tcb200.h"

static char* slurp(const char* path, long* n) {
  FILE* f = fopen(path, "rb");
  if (!f) { perror(path); exit(2); }
  fseek(f, 0, SEEK_END);
  *n = ftell(f);
  fseek(f, 0, SEEK_SET);
  char* b = (char*)malloc((size_t)*n + 1);
  if (fread(b, 1, (size_t)*n, f) != (size_t)*n) { perror(path); exit(2); }
  b[*n] = 0;
  fclose(f);
  return b;
}

/* Node sizes and whether each node is an input: scans the top-level "nodes" array for each node's
 * "op" and its last "shape" entry (a node's own shape follows its attrs in Graph.toJSON's order). */
static int scan_nodes(const char* js, int64_t* sizes, int* is_input, int cap) {
  int n = 0, depth = 0;
  const char* p = strstr(js, "\"nodes\"");
  p = strchr(p, '[');
  const char* node_start = NULL;
  for (; *p; ++p) {
    if (*p == '{' || *p == '[') {
      if (depth == 1 && *p == '{') node_start = p;
      depth++;
    } else if (*p == '}' || *p == ']') {
      depth--;
      if (depth == 1 && *p == '}') {
        /* one top-level node spans node_start .. p: its op and its final "shape" list */
        const char* op = strstr(node_start, "\"op\"");
        op = strchr(op + 4, '"');
        is_input[n] = strncmp(op, "\"input\"", 7) == 0;
        const char* last = NULL;
        for (const char* q = node_start; q < p; ++q)
          if (strncmp(q, "\"shape\"", 7) == 0) last = q;
        int64_t s = 1;
        const char* q = strchr(last, '[') + 1;
        while (*q != ']') {
          s *= strtoll(q, (char**)&q, 10);
          while (*q == ',' || *q == ' ') ++q;
        }
        sizes[n++] = s;
        if (n == cap) return n;
      }
      if (depth == 0) break;
    }
  }
  return n;
}

int main(int argc, char** argv) {
  if (argc != 5) { fprintf(stderr, "usage: run_graph GRAPH.json OPTS.json INPUTS.bin OUT.bin\n"); return 2; }
  long ng, no, ni;
  char* graph = slurp(argv[1], &ng);
  char* opts = slurp(argv[2], &no);
  char* inbin = slurp(argv[3], &ni);
  enum { CAP = 1 << 16 };
  static int64_t sizes[CAP];
  static int is_input[CAP];
  int n = scan_nodes(graph, sizes, is_input, CAP);
  tc_lowered* low = NULL;
  if (tc_lower_json(graph, opts, &low)) { fprintf(stderr, "lower: %s\n", tc_last_error()); return 1; }
  int launches = 0;
  tc_lowered_count(low, &launches);
  const float** ins = (const float**)calloc((size_t)n, sizeof(float*));
  float** vals = (float**)calloc((size_t)n, sizeof(float*));
  int* intact = (int*)calloc((size_t)n, sizeof(int));
  long off = 0;
  for (int i = 0; i < n; ++i) {
    if (is_input[i]) { ins[i] = (const float*)(inbin + off); off += sizes[i] * 4; }
    vals[i] = (float*)malloc((size_t)(sizes[i] ? sizes[i] : 1) * 4);
  }
  if (off != ni) { fprintf(stderr, "inputs: %ld bytes given, %ld needed\n", ni, off); return 2; }
  tc_ctx* ctx = NULL;
  if (tc_open(0, &ctx)) { fprintf(stderr, "open: %s\n", tc_last_error()); return 1; }
  if (tc_lowered_run(ctx, low, ins, vals, 1, intact)) { fprintf(stderr, "run: %s\n", tc_last_error()); return 1; }
  FILE* f = fopen(argv[4], "wb");
  for (int i = 0; i < n; ++i) {
    if (!intact[i]) { fprintf(stderr, "node %d wrote past its buffer\n", i); return 1; }
    fwrite(vals[i], 4, (size_t)sizes[i], f);
  }
  fclose(f);
  tc_close(ctx);
  tc_lowered_free(low);
  printf("{\"nodes\": %d, \"launches\": %d}\n", n, launches);
  return 0;
}
