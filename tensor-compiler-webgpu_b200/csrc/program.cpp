// program.cpp -- running a lowering made by tc_lower_json, with no host language between the caller
// and the library: the verification runner and the trainers' resident program.
//
//  * tc_lowered_run is GpuRunner.run (src/gpu/runtime.js:60-129): a buffer per node, canary-padded
//    when asked, inputs and constants uploaded, every launch issued in order (a tensor-core launch's
//    bounded-wait error word checked after it), every requested node read back.
//  * tc_program_* is the persistent step of GpuTrainer / FusedTrainer (src/gpu/trainer.js:13-104,
//    src/fusion/trainer-fused.js:135-213): inputs, constants, kept values and feedback ends own
//    buffers; every other value lives in one arena at an offset from tc_plan_memory (lifetime best
//    fit); a plain reshape shares its source's memory; a launch no kept or fed-back value depends on
//    is left out; the launches, then the feedback copies, replay from one native plan (one CUDA graph
//    once captured).  Values are those of the runner, bit for bit.
//
// Kernels come from the on-disk cache the Python host fills (file = first 32 hex digits of the SHA-256
// of the source, a NUL and the decimal template hash; directory $TCB_KERNEL_CACHE, else _kernel_cache
// beside this library), compiled by NVRTC on a miss and written back.
#include <dlfcn.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>

#include "lower.h"

namespace tcb_detail {
int fail_msg(int status, const std::string& msg);
}

namespace {

// ---------------------------------------------------------------- SHA-256 (FIPS 180-4)
struct Sha256 {
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  uint64_t len = 0;
  unsigned char buf[64];
  size_t fill = 0;

  static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

  void block(const unsigned char* p) {
    static const uint32_t K[64] = {
        0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5, 0xd807aa98,
        0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786,
        0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8,
        0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13,
        0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819,
        0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a,
        0x5b9cca4f, 0x682e6ff3, 0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
        0xc67178f2};
    uint32_t w[64];
    for (int i = 0; i < 16; ++i) w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      uint32_t ch = (e & f) ^ (~e & g);
      uint32_t t1 = hh + S1 + ch + K[i] + w[i];
      uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
      uint32_t t2 = S0 + mj;
      hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  void update(const void* data, size_t n) {
    const unsigned char* p = static_cast<const unsigned char*>(data);
    len += n;
    while (n) {
      size_t k = std::min(n, 64 - fill);
      memcpy(buf + fill, p, k);
      fill += k; p += k; n -= k;
      if (fill == 64) { block(buf); fill = 0; }
    }
  }
  std::string hex() {
    uint64_t bits = len * 8;
    unsigned char pad = 0x80;
    update(&pad, 1);
    unsigned char z = 0;
    while (fill != 56) update(&z, 1);
    unsigned char L[8];
    for (int i = 0; i < 8; ++i) L[i] = (unsigned char)(bits >> (56 - 8 * i));
    update(L, 8);
    char out[65];
    for (int i = 0; i < 8; ++i) snprintf(out + 8 * i, 9, "%08x", h[i]);
    return std::string(out, 64);
  }
};

std::string cache_dir() {
  if (const char* e = getenv("TCB_KERNEL_CACHE")) return e;
  Dl_info info;
  if (dladdr(reinterpret_cast<void*>(&tc_lowered_run), &info) && info.dli_fname) {
    std::string p = info.dli_fname;
    size_t s = p.rfind('/');
    return (s == std::string::npos ? std::string(".") : p.substr(0, s)) + "/_kernel_cache";
  }
  return "_kernel_cache";
}

std::mutex g_cubin_mu;
std::map<std::string, std::vector<char>> g_cubins;   // source -> cubin (process-wide; cubins are device-independent)

int cubin_for(const std::string& code, const std::vector<char>** out) {
  {
    std::lock_guard<std::mutex> lock(g_cubin_mu);
    auto it = g_cubins.find(code);
    if (it != g_cubins.end()) {
      *out = &it->second;
      return TC_OK;
    }
  }
  Sha256 sh;
  sh.update(code.data(), code.size());
  unsigned char nul = 0;
  sh.update(&nul, 1);
  std::string th = std::to_string(tc_templates_hash());
  sh.update(th.data(), th.size());
  std::string path = cache_dir() + "/" + sh.hex().substr(0, 32) + ".cubin";
  std::vector<char> data;
  std::ifstream f(path, std::ios::binary);
  if (f) {
    data.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  } else {
    uint64_t n = 0;
    std::vector<char> log(1 << 16);
    if (int s = tc_compile_cubin(code.c_str(), nullptr, 0, &n, log.data(), log.size())) return s;
    data.resize(n);
    if (int s = tc_compile_cubin(code.c_str(), data.data(), n, &n, log.data(), log.size())) return s;
    data.resize(n);
    std::string tmp = path + "." + std::to_string(getpid()) + ".tmp";
    mkdir(cache_dir().c_str(), 0755);
    std::ofstream o(tmp, std::ios::binary);
    if (o) {
      o.write(data.data(), (std::streamsize)data.size());
      o.close();
      rename(tmp.c_str(), path.c_str());
    }
  }
  std::lock_guard<std::mutex> lock(g_cubin_mu);
  auto& slot = g_cubins[code];
  slot = std::move(data);
  *out = &slot;
  return TC_OK;
}

int module_for(tc_ctx* ctx, const std::string& code, tc_module** mod) {
  const std::vector<char>* cubin = nullptr;
  if (int s = cubin_for(code, &cubin)) return s;
  return tc_module_load(ctx, cubin->data(), cubin->size(), mod);
}

}  // namespace

// ---------------------------------------------------------------- issuing one call
namespace {

using tcl::Call;
using tcl::Launch;
using tcl::i64;

i64 info_int(const Launch& l, const char* key, i64 dflt) {
  for (auto& kv : l.info)
    if (kv.first == key && kv.second.is_number()) return kv.second.as_int();
  return dflt;
}

// The argument block and tensor-map descriptors of one call (the Python host's runtime.issue).
struct Issued {
  tc_args args;
  std::vector<uint64_t> desc;
};

int prepare_call(const Call& c, const std::vector<uint64_t>& ins, uint64_t out, uint64_t scratch, uint64_t err_ptr,
                 const std::map<int, uint64_t>& ptrs, Issued* is) {
  memset(&is->args, 0, sizeof is->args);
  std::vector<i64> params = c.params;
  if (c.out_node >= 0) {
    auto it = ptrs.find(c.out_node);
    if (it == ptrs.end()) return tcb_detail::fail_msg(TC_ERR_INVALID, "call " + c.name + ": second output has no buffer");
    out = it->second;
  }
  for (auto& pp : c.ptr_params) {
    auto it = ptrs.find(pp.second);
    if (it == ptrs.end()) return tcb_detail::fail_msg(TC_ERR_INVALID, "call " + c.name + ": second output has no buffer");
    while ((int)params.size() <= pp.first) params.push_back(0);
    params[pp.first] = (i64)it->second;
  }
  if (c.err_offset >= 0) {
    while (params.size() < 16) params.push_back(0);
    params[15] = (i64)(err_ptr ? err_ptr : scratch + (uint64_t)c.err_offset);
  }
  if (ins.size() > TC_MAX_OPERANDS || params.size() > TC_MAX_PARAMS)
    return tcb_detail::fail_msg(TC_ERR_INVALID, "call " + c.name + ": too many operands or parameters");
  for (size_t k = 0; k < ins.size(); ++k) is->args.in[k] = ins[k];
  is->args.out = out;
  is->args.scratch = scratch;
  for (size_t k = 0; k < params.size(); ++k) is->args.p[k] = params[k];
  is->desc.clear();
  for (auto& m : c.tma) {
    uint64_t addr;
    if (m.region == "scratch") addr = scratch + (uint64_t)m.off;
    else if (m.region == "in") addr = ins.at((size_t)m.off);
    else if (m.region == "out") addr = out + (uint64_t)m.off;
    else return tcb_detail::fail_msg(TC_ERR_INVALID, "tensor map over '" + m.region + "'");
    if (addr % 16) return tcb_detail::fail_msg(TC_ERR_INVALID, "call " + c.name + ": tensor map base is not 16-byte aligned");
    uint64_t v[8] = {addr, (uint64_t)m.cols, (uint64_t)m.rows, (uint64_t)m.batches, (uint64_t)m.rs, (uint64_t)m.bs,
                     (uint64_t)m.bc, (uint64_t)m.br};
    is->desc.insert(is->desc.end(), v, v + 8);
  }
  return TC_OK;
}

void dims(const Call& c, uint32_t g[3], uint32_t b[3]) {
  for (int k = 0; k < 3; ++k) {
    g[k] = (uint32_t)c.grid[k];
    b[k] = (uint32_t)c.block[k];
  }
}

int launch_now(tc_module* mod, const Call& c, const Issued& is) {
  uint32_t g[3], b[3];
  dims(c, g, b);
  if (c.has_tma)
    return tc_launch_tma(mod, c.name.c_str(), g, b, (uint32_t)c.smem, (int)c.tma.size(), is.desc.data(), &is.args);
  return tc_launch(mod, c.name.c_str(), g, b, (uint32_t)c.smem, &is.args);
}

int plan_add(tc_plan* plan, tc_module* mod, const Call& c, const Issued& is) {
  uint32_t g[3], b[3];
  dims(c, g, b);
  if (c.has_tma)
    return tc_plan_add_launch_tma(plan, mod, c.name.c_str(), g, b, (uint32_t)c.smem, (int)c.tma.size(), is.desc.data(),
                                  &is.args);
  return tc_plan_add_launch(plan, mod, c.name.c_str(), g, b, (uint32_t)c.smem, &is.args);
}

struct Bufs {
  std::vector<tc_buf*> all;
  ~Bufs() {
    for (auto* b : all) tc_free(b);
  }
  int alloc(tc_ctx* ctx, uint64_t bytes, uint64_t canary, tc_buf** out) {
    if (int s = tc_alloc(ctx, bytes, canary, out)) return s;
    all.push_back(*out);
    return TC_OK;
  }
};

uint64_t ptr_of(tc_buf* b) {
  uint64_t p = 0;
  tc_buf_ptr(b, &p);
  return p;
}

int upload_const(tc_ctx* ctx, const tcl::Node& n, uint64_t dst) {
  i64 count = 1;
  for (i64 d : n.shape) count *= d;
  std::vector<float> v((size_t)std::max<i64>(count, 1));
  for (i64 i = 0; i < count; ++i) v[(size_t)i] = (float)(n.scalar_value ? n.value : n.values.at((size_t)i));
  if (count == 0) return TC_OK;
  return tc_memcpy_htod(ctx, dst, v.data(), (uint64_t)count * 4);
}

i64 nsize(const tcl::Node& n) {
  i64 c = 1;
  for (i64 d : n.shape) c *= d;
  return c;
}

}  // namespace

extern "C" {

int tc_lowered_run(tc_ctx* ctx, tc_lowered* l, const float* const* inputs, float* const* values, int canary,
                   int* canary_intact) {
  if (!ctx || !l) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_lowered_run: null argument");
  const tcl::Graph& g = *l->L.graph;
  const int WGs = 256;
  Bufs bufs;
  std::vector<tc_buf*> nb(g.nodes.size(), nullptr);
  std::map<int, uint64_t> ptrs;
  for (auto& n : g.nodes) {
    i64 c = nsize(n);
    uint64_t pad = canary ? (uint64_t)((((c + WGs - 1) / WGs) * WGs + WGs - c) * 4) : 0;
    if (int s = bufs.alloc(ctx, (uint64_t)std::max<i64>(1, c) * 4, pad, &nb[n.id])) return s;
    ptrs[n.id] = ptr_of(nb[n.id]);
  }
  for (auto& n : g.nodes) {
    if (n.op == "input") {
      if (!inputs || !inputs[n.id])
        return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_lowered_run: no value for input '" + n.name + "'");
      if (nsize(n))
        if (int s = tc_upload(nb[n.id], inputs[n.id], (uint64_t)nsize(n) * 4, 0)) return s;
    } else if (n.op == "const") {
      if (int s = upload_const(ctx, n, ptrs[n.id])) return s;
    }
  }
  i64 scratch_bytes = 0;
  for (auto& lau : l->L.launches) scratch_bytes = std::max(scratch_bytes, lau.scratch_bytes);
  tc_buf* sbuf = nullptr;
  uint64_t scratch = 0;
  if (scratch_bytes > 0) {
    if (int s = bufs.alloc(ctx, (uint64_t)scratch_bytes, 0, &sbuf)) return s;
    scratch = ptr_of(sbuf);
    if (int s = tc_memset32(ctx, scratch, 0, (uint64_t)scratch_bytes / 4)) return s;   // error words start clear
  }
  Issued is;
  for (auto& lau : l->L.launches) {
    tc_module* mod = nullptr;
    if (int s = module_for(ctx, lau.code, &mod)) return s;
    std::vector<uint64_t> ins;
    for (int i : lau.inputs) ins.push_back(ptrs[i]);
    bool waits = false;
    for (auto& c : lau.calls) {
      if (int s = prepare_call(c, ins, ptrs[lau.node], lau.scratch_bytes ? scratch : 0, 0, ptrs, &is)) return s;
      if (int s = launch_now(mod, c, is)) return s;
      waits |= c.err_offset >= 0;
    }
    if (waits) {
      if (int s = tc_sync(ctx, 600000)) return s;
      for (auto& c : lau.calls) {
        if (c.err_offset < 0) continue;
        uint32_t w = 0;
        if (int s = tc_memcpy_dtoh(ctx, &w, scratch + (uint64_t)c.err_offset, 4)) return s;
        if (int s = tc_sync(ctx, 600000)) return s;
        if (w) {
          tc_memset32(ctx, scratch + (uint64_t)c.err_offset, 0, 1);
          return tcb_detail::fail_msg(TC_ERR_TIMEOUT, c.name + ": a bounded wait ran out (code " + std::to_string(w) + ")");
        }
      }
    }
  }
  if (int s = tc_sync(ctx, 600000)) return s;
  for (auto& n : g.nodes) {
    if (values && values[n.id] && nsize(n))
      if (int s = tc_download(nb[n.id], values[n.id], (uint64_t)nsize(n) * 4, 0)) return s;
    if (canary && canary_intact) {
      int ok = 0;
      if (int s = tc_check_canary(nb[n.id], &ok)) return s;
      canary_intact[n.id] = ok;
    }
  }
  return TC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- the resident program
struct tc_program {
  tc_ctx* ctx = nullptr;
  const tc_lowered* lowered = nullptr;
  std::vector<tc_buf*> bufs;
  std::map<int, uint64_t> ptrs;
  std::vector<int> err_words;   // byte offsets of the launches' error words in `errs`
  tc_buf* errs = nullptr;
  uint64_t errs_ptr = 0;
  tc_plan* plan = nullptr;
  int launches = 0;
  ~tc_program() {
    if (plan) tc_plan_free(plan);
    for (auto* b : bufs) tc_free(b);
  }
};

extern "C" {

int tc_program_create(tc_ctx* ctx, tc_lowered* l, const int32_t* keep, int n_keep, const int32_t* feedback,
                      int n_feedback, int capture, tc_program** out) {
  if (!ctx || !l || !out || (n_keep && !keep) || (n_feedback && !feedback))
    return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_create: null argument");
  *out = nullptr;
  const tcl::Graph& g = *l->L.graph;
  const int N = (int)g.nodes.size();
  auto bad = [&](int id) { return id < 0 || id >= N; };
  std::set<int> kept, fb;
  for (int k = 0; k < n_keep; ++k) {
    if (bad(keep[k])) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_create: keep id out of range");
    kept.insert(keep[k]);
  }
  std::vector<std::pair<int, int>> pairs;
  for (int k = 0; k < n_feedback; ++k) {
    int a = feedback[2 * k], b = feedback[2 * k + 1];
    if (bad(a) || bad(b)) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_create: feedback id out of range");
    pairs.emplace_back(a, b);
    fb.insert(a);
    fb.insert(b);
  }
  auto p = std::make_unique<tc_program>();
  p->ctx = ctx;
  p->lowered = l;
  // values something kept or fed back depends on
  std::set<int> live(kept.begin(), kept.end());
  for (auto& pr : pairs) live.insert(pr.first);
  for (int i = N - 1; i >= 0; --i)
    if (live.count(i))
      for (int j : g.nodes[i].inputs) live.insert(j);
  std::map<int, int> alias;   // a plain reshape shares its source's memory
  std::vector<const Launch*> launches;
  for (auto& lau : l->L.launches) {
    std::vector<int> outs = lau.nodes.empty() ? std::vector<int>{lau.node} : lau.nodes;
    bool any = false;
    for (int o : outs) any |= live.count(o) > 0;
    if (!any) continue;
    const tcl::Node& n = g.nodes[lau.node];
    if (n.op == "reshape" && lau.kind == "gather" && !kept.count(lau.node) && !fb.count(lau.node)) {
      alias[lau.node] = lau.inputs[0];
      continue;
    }
    launches.push_back(&lau);
  }
  auto root = [&](int i) {
    while (alias.count(i)) i = alias[i];
    return i;
  };
  std::map<int, int> first, last;
  for (int k = 0; k < (int)launches.size(); ++k) {
    const Launch& lau = *launches[k];
    std::vector<int> outs = lau.nodes.empty() ? std::vector<int>{lau.node} : lau.nodes;
    for (int o : outs) first[o] = k;
    for (int i : lau.inputs) {
      int r = root(i);
      last[r] = std::max(last.count(r) ? last[r] : -1, k);
    }
  }
  std::vector<int> arena_ids;
  for (auto& n : g.nodes) {
    if (alias.count(n.id)) continue;
    uint64_t nbytes = (uint64_t)std::max<i64>(1, nsize(n)) * 4;
    bool own = n.op == "input" || n.op == "const" || kept.count(n.id) || fb.count(n.id) ||
               (!first.count(n.id) && last.count(n.id));
    if (own) {
      tc_buf* b = nullptr;
      if (int s = tc_alloc(ctx, nbytes, 0, &b)) return s;
      p->bufs.push_back(b);
      p->ptrs[n.id] = ptr_of(b);
      if (n.op == "const")
        if (int s = upload_const(ctx, n, p->ptrs[n.id])) return s;
    } else if (first.count(n.id)) {
      arena_ids.push_back(n.id);
    }
  }
  if (!arena_ids.empty()) {
    std::vector<uint64_t> bytes, offs(arena_ids.size());
    std::vector<int32_t> f, la;
    for (int id : arena_ids) {
      bytes.push_back((uint64_t)std::max<i64>(1, nsize(g.nodes[id])) * 4);
      f.push_back(first[id]);
      la.push_back(last.count(id) ? last[id] : first[id]);
    }
    uint64_t total = 0;
    if (int s = tc_plan_memory((int)arena_ids.size(), bytes.data(), f.data(), la.data(), offs.data(), &total)) return s;
    tc_buf* arena = nullptr;
    if (int s = tc_alloc(ctx, std::max<uint64_t>(total, 256), 0, &arena)) return s;
    p->bufs.push_back(arena);
    uint64_t base = ptr_of(arena);
    for (size_t k = 0; k < arena_ids.size(); ++k) p->ptrs[arena_ids[k]] = base + offs[k];
  }
  for (auto& a : alias) p->ptrs[a.first] = p->ptrs[root(a.first)];
  i64 scratch_bytes = 0;
  for (auto* lau : launches) scratch_bytes = std::max(scratch_bytes, lau->scratch_bytes);
  uint64_t scratch = 0;
  if (scratch_bytes) {
    tc_buf* sb = nullptr;
    if (int s = tc_alloc(ctx, (uint64_t)scratch_bytes, 0, &sb)) return s;
    p->bufs.push_back(sb);
    scratch = ptr_of(sb);
    if (int s = tc_memset32(ctx, scratch, 0, (uint64_t)scratch_bytes / 4)) return s;
  }
  // a private control block (error word + split-tile arrival counters) per launch with a bounded wait:
  // the blocks start zeroed and return to zero after every run, so no clearing launch is planned
  std::vector<uint64_t> slot(launches.size(), 0);
  uint64_t off = 0;
  for (size_t k = 0; k < launches.size(); ++k) {
    bool has = false;
    for (auto& c : launches[k]->calls) has |= c.err_offset >= 0;
    if (has) {
      slot[k] = off + 1;
      p->err_words.push_back((int)off);
      off += (uint64_t)info_int(*launches[k], "ctrl_bytes", 64);
    }
  }
  uint64_t errs_bytes = std::max<uint64_t>(64, off);
  if (int s = tc_alloc(ctx, errs_bytes, 0, &p->errs)) return s;
  p->bufs.push_back(p->errs);
  p->errs_ptr = ptr_of(p->errs);
  if (int s = tc_memset32(ctx, p->errs_ptr, 0, errs_bytes / 4)) return s;
  if (int s = tc_plan_create(ctx, &p->plan)) return s;
  Issued is;
  for (size_t k = 0; k < launches.size(); ++k) {
    const Launch& lau = *launches[k];
    tc_module* mod = nullptr;
    if (int s = module_for(ctx, lau.code, &mod)) return s;
    std::vector<uint64_t> ins;
    for (int i : lau.inputs) ins.push_back(p->ptrs.at(i));
    for (auto& c : lau.calls) {
      if (c.name == "tcb_gemm_prep") continue;   // the private control block needs no clearing launch
      uint64_t err = slot[k] ? p->errs_ptr + slot[k] - 1 : 0;
      if (int s = prepare_call(c, ins, p->ptrs.at(lau.node), lau.scratch_bytes ? scratch : 0, err, p->ptrs, &is)) return s;
      if (int s = plan_add(p->plan, mod, c, is)) return s;
      p->launches++;
    }
  }
  for (auto& pr : pairs) {
    uint64_t n = (uint64_t)std::max<i64>(1, nsize(g.nodes[pr.second])) * 4;
    if (int s = tc_plan_add_copy(p->plan, p->ptrs.at(pr.second), p->ptrs.at(pr.first), n)) return s;
  }
  if (capture)
    if (int s = tc_plan_capture(p->plan)) return s;
  *out = p.release();
  return TC_OK;
}

int tc_program_ptr(tc_program* p, int node, uint64_t* dptr) {
  if (!p || !dptr) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_ptr: null argument");
  auto it = p->ptrs.find(node);
  if (it == p->ptrs.end())
    return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_ptr: node " + std::to_string(node) + " has no memory in this program");
  *dptr = it->second;
  return TC_OK;
}

int tc_program_write(tc_program* p, int node, const float* host, uint64_t count) {
  uint64_t d = 0;
  if (int s = tc_program_ptr(p, node, &d)) return s;
  const tcl::Node& n = p->lowered->L.graph->nodes.at((size_t)node);
  if ((i64)count != nsize(n))
    return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_write: node " + std::to_string(node) + " holds " +
                                                    std::to_string(nsize(n)) + " values, " + std::to_string(count) + " given");
  if (int s = tc_memcpy_htod(p->ctx, d, host, count * 4)) return s;
  return tc_sync(p->ctx, 600000);
}

int tc_program_read(tc_program* p, int node, float* host, uint64_t count) {
  uint64_t d = 0;
  if (int s = tc_program_ptr(p, node, &d)) return s;
  const tcl::Node& n = p->lowered->L.graph->nodes.at((size_t)node);
  if ((i64)count != nsize(n))
    return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_read: node " + std::to_string(node) + " holds " +
                                                    std::to_string(nsize(n)) + " values, " + std::to_string(count) + " asked");
  if (int s = tc_sync(p->ctx, 600000)) return s;
  if (int s = tc_memcpy_dtoh(p->ctx, host, d, count * 4)) return s;
  return tc_sync(p->ctx, 600000);
}

int tc_program_run(tc_program* p) {
  if (!p) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_run: null program");
  return tc_plan_run(p->plan);
}

int tc_program_check(tc_program* p) {
  if (!p) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_check: null program");
  if (p->err_words.empty()) return TC_OK;
  if (int s = tc_sync(p->ctx, 600000)) return s;
  for (int off : p->err_words) {
    uint32_t w = 0;
    if (int s = tc_memcpy_dtoh(p->ctx, &w, p->errs_ptr + (uint64_t)off, 4)) return s;
    if (int s = tc_sync(p->ctx, 600000)) return s;
    if (w) {
      tc_memset32(p->ctx, p->errs_ptr + (uint64_t)off, 0, 1);
      return tcb_detail::fail_msg(TC_ERR_TIMEOUT, "a tensor-core launch's bounded wait ran out (code " + std::to_string(w) + ")");
    }
  }
  return TC_OK;
}

int tc_program_launch_count(tc_program* p, int* n) {
  if (!p || !n) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_program_launch_count: null argument");
  *n = p->launches;
  return TC_OK;
}

int tc_program_free(tc_program* p) {
  delete p;
  return TC_OK;
}

}  // extern "C"
