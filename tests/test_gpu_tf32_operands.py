"""How the tensor cores read an fp32 operand of a kind::tf32 MMA (an in-bounds check on a correct GEMM).

The GEMM kernel is run with its split passes replaced by copies that put the raw fp32 value in the
"hi" operand and zero in "lo", with B = 1 and bias 0, so each output is the sum over k of what the
tensor core made of A[i, k].  Three bit patterns tell truncation, round-half-away and round-half-even
apart: 1 + 2^-12 (below half an ulp of tf32), 1 + 2^-11 (exactly half), 1 + 2^-11 + 2^-12 (above).
The in-kernel operand split relies on the answer: it uses the raw value as hi and x - tf32(x) as lo.
"""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PROBE = r"""
extern "C" __global__ void probe_split_a(const tcb::Args a) {
  float* hi = reinterpret_cast<float*>(a.scratch);
  float* lo = hi + (u64)TCB_BATCH * TCB_M * TCB_KP;
  const float* src = reinterpret_cast<const float*>(a.in[TCB_IA]);
  for (u64 i = (u64)blockIdx.x * blockDim.x + threadIdx.x; i < (u64)TCB_M * TCB_KP; i += (u64)gridDim.x * blockDim.x) {
    const u64 r = i / TCB_KP, k = i % TCB_KP;
    hi[i] = k < TCB_K ? src[r * TCB_K + k] : 0.0f;
    lo[i] = 0.0f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.p[15]) *reinterpret_cast<u32*>(a.p[15]) = 0u;
}
extern "C" __global__ void probe_split_b(const tcb::Args a) {
  float* hi = reinterpret_cast<float*>(a.scratch) + 2ull * TCB_BATCH * TCB_M * TCB_KP;
  float* lo = hi + (u64)TCB_BATCH * TCB_N * TCB_KP;
  for (u64 i = (u64)blockIdx.x * blockDim.x + threadIdx.x; i < (u64)TCB_N * TCB_KP; i += (u64)gridDim.x * blockDim.x) {
    hi[i] = (i % TCB_KP) < TCB_K ? 1.0f : 0.0f;
    lo[i] = 0.0f;
  }
}
"""


def test_tf32_operand_bits(pkg, runner, monkeypatch):
    monkeypatch.setenv("TCB_GEMM_FUSED", "0")   # the launch with split passes, whose splits the probe replaces
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    M, K, N = 128, 32, 128
    W = wl.c3_graph(M, K, N, "relu")
    fused = pkg.fuse.fuse(W["graph"], keep=W["keep"])
    lau = next(l for l in cg.lower_fused(fused.graph, matmul="tiled")["launches"] if l.calls[-1].name == "tcb_gemm_tc")
    mod = runner.pipeline(lau.code + PROBE)
    pats = np.array([0x3F800800, 0x3F801000, 0x3F801800, 0x3F800000], dtype=np.uint32)  # 1+2^-12, 1+2^-11, 1+2^-11+2^-12, 1
    a = np.repeat(pats, M // 4)[:, None].repeat(K, axis=1).view(np.float32)
    bufs = {"a": a, "b": np.ones((K, N), np.float32), "bias": np.zeros(N, np.float32)}
    node_name = {n.id: n.attrs["name"] for n in fused.graph.nodes if n.op == "input"}
    dev = {}
    out = rt.DeviceBuffer(runner, M * N * 4)
    try:
        for nid in lau.inputs:
            arr = bufs[node_name[nid]]
            dev[nid] = rt.DeviceBuffer(runner, arr.nbytes)
            dev[nid].upload(arr)
        scratch = runner.scratch(lau.scratch_bytes)
        calls = [c for c in lau.calls]
        calls[0].name, calls[1].name = "probe_split_a", "probe_split_b"
        calls[0].grid, calls[1].grid = (16, 1, 1), (16, 1, 1)
        for c in calls:
            rt.issue(c, mod, [dev[nid].ptr for nid in lau.inputs], out.ptr, scratch)
        runner.sync()
        runner.check_errors(lau, scratch)
        y = out.download(M * N).reshape(M, N)
    finally:
        for b in dev.values():
            b.free()
        out.free()
    got = [float(y[q * (M // 4), 0]) for q in range(4)]
    trunc = [32.0, 32.0, 32.0, 32.0]
    rna = [32.0, 32.0 * (1 + 2 ** -10), 32.0 * (1 + 2 ** -10), 32.0]
    rne = [32.0, 32.0, 32.0 * (1 + 2 ** -10), 32.0]
    kind = {tuple(trunc): "truncate", tuple(rna): "round-half-away", tuple(rne): "round-half-even"}.get(tuple(got))
    print("tf32 operand read:", kind, got)
    assert kind == "truncate", got
