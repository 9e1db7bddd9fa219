// Fusions found while a compiled function is recorded (shlo_compile with
// enable = 1; MLX's mx::compile fuses in the same place in the reference,
// c/smlx_shim.c:360-374).
//
// The recording calls the traced function twice on the same private inputs:
// once eagerly, then inside the CUDA-graph capture. During the eager call every
// entry point that reads array data logs itself (kind, parameter words, the
// layouts and storage of its inputs, the storage of its result). From that log
// the recorder finds op chains whose intermediate results nothing else reads
// and that one of the library's fused kernels computes with the same
// roundings, in the same order:
//
//   dense      mul_mat (one weight, no batch) -> add of a broadcast 1-D bias over
//              the last axis [-> add of a same-shape residual] [-> gelu_erf]:
//              k_mul_mat_fused (Lower.lean:157-182's dot_general followed by
//              the module's adds)
//   layer norm norm -> multiply by a broadcast 1-D gain -> add a broadcast 1-D
//              bias: k_norm_affine
//   attention  the copies of q and k into [batch*head*position, 64], the scores
//              mul_mat, soft_max, the copy of v, the value mul_mat, and the copy
//              of the result into [batch, position, head*64]: k_attention
//
// A dense chain ending in gelu_erf, an attention block or a layer norm whose
// result only the next dense chain's product reads, as its whole x, writes it
// in that product's packed x layout, so the product skips its pack.
//
// In the capture call the same entry points are matched to the log op by op.
// An op inside a chain returns a placeholder of the logged shape (real storage
// that nothing writes or reads) and the chain's last op launches the fused
// kernel on the handles the chain's ops received. If the second call departs
// from the log in any way, the recording is dropped and the function runs
// eagerly, unfused, for that signature. The eager path (enable = 0) never
// fuses. $SHLO_FUSE=0 turns the fusions off.
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"

namespace shlo {

thread_local Tracer *t_tracer = nullptr;
thread_local int t_trace_depth = 0;

namespace {

enum { ROLE_NONE = -1 };
enum GroupKind { G_DENSE = 1, G_NORM, G_ATTN };
// roles inside a chain
enum { R_MM = 0, R_BIAS, R_RES, R_GELU, R_NORM = 0, R_GAIN, R_BETA, R_CQ = 0, R_CK, R_SCORES, R_SOFTMAX, R_CV, R_VALUE, R_COPY_OUT };

struct TIn {
  uint64_t buf = 0;  // storage serial (0: no storage)
  uint8_t dtype = 0;
  int ndim = 0;
  int64_t offset = 0;
  int64_t shape[kMaxRank] = {0};
  int64_t strides[kMaxRank] = {0};
};

struct TOp {
  int kind = 0, sub = 0;
  uint32_t p[8] = {0};
  int np = 0;
  std::vector<TIn> in;
  uint64_t out = 0;
  uint8_t out_dtype = 0;
  int out_ndim = 0;
  int64_t out_shape[kMaxRank] = {0};
};

struct Group {
  int kind = 0;
  std::vector<int> ops;  // log indices, in order
  int last = -1;
  int flags = 0;         // dense: the epilogue flags
  int direct = 0;        // attention: q (1), k (2), v (4) read directly, without a copy
  uint32_t p[8] = {0};   // the fused kernel's parameter words
  // chains linked through a packed operand: y_pack (this chain's result is the
  // next dense chain's x, written in its packed layout) and x_np (this dense
  // chain's x is an earlier chain's result, already packed; src is that chain)
  int y_pack[2] = {0, 0};
  int x_np = 0, src = -1;
  uint64_t produced = 0;  // the capture call: the serial of the fused result's storage
  // the capture call's handles, retained until the fused launch
  Arr *h[4] = {nullptr, nullptr, nullptr, nullptr};
  std::map<int, Buffer *> placeholder;  // role -> its placeholder storage
  bool done = false;
};

TIn in_of(const Arr *a) {
  TIn t;
  t.buf = a->buf ? a->buf->serial : 0;
  t.dtype = a->dtype;
  t.ndim = a->ndim;
  t.offset = a->offset;
  for (int i = 0; i < a->ndim; i++) {
    t.shape[i] = a->shape[i];
    t.strides[i] = a->strides[i];
  }
  return t;
}

int64_t count_of(const TIn &t) {
  int64_t n = 1;
  for (int i = 0; i < t.ndim; i++) n *= t.shape[i];
  return n;
}

bool row_major(const TIn &t) {
  int64_t s = 1;
  for (int i = t.ndim - 1; i >= 0; i--) {
    if (t.shape[i] != 1 && t.strides[i] != s) return false;
    s *= t.shape[i];
  }
  return true;
}

// All of storage `buf`'s first `count` f32 values, in row-major order.
bool full_view(const TIn &t, uint64_t buf, int64_t count) {
  return t.buf == buf && buf != 0 && t.dtype == kF32 && t.offset == 0 && row_major(t) && count_of(t) == count;
}

// A 1-D vector of `m` f32 values broadcast over every axis but the last.
bool bcast_last(const TIn &t, int64_t m, int ndim, const int64_t *shape) {
  if (t.dtype != kF32 || t.ndim != ndim || ndim < 1 || t.buf == 0) return false;
  for (int i = 0; i < ndim; i++)
    if (t.shape[i] != shape[i]) return false;
  if (t.shape[ndim - 1] != m || (m > 1 && t.strides[ndim - 1] != 1)) return false;
  for (int i = 0; i < ndim - 1; i++)
    if (t.shape[i] != 1 && t.strides[i] != 0) return false;
  return true;
}

bool same_layout(const TIn &a, const TIn &b) {
  if (a.dtype != b.dtype || a.ndim != b.ndim || a.offset != b.offset) return false;
  for (int i = 0; i < a.ndim; i++)
    if (a.shape[i] != b.shape[i] || a.strides[i] != b.strides[i]) return false;
  return true;
}

// A contiguous, 16-byte-aligned version of `a` (what shlo_kernel_apply hands the kernels).
int prep(Device *dev, Arr *a, Arr **out) {
  Arr *c;
  SHLO_TRY(make_contiguous(a, &c));
  if (c->buf && ((uintptr_t)data_ptr(c) & 15)) {
    Arr *d = nullptr;
    int rc = new_array(dev, c->dtype, c->shape, c->ndim, &d);
    if (!rc) rc = launch_copy_strided(dev, c, d->buf->ptr);
    shlo_release(c);
    if (rc) {
      if (d) shlo_release(d);
      return 1;
    }
    c = d;
  }
  *out = c;
  return 0;
}

// A view of `a` with its axes permuted (out axis i = a's axis perm[i]).
Arr *permuted(const Arr *a, const int *perm) {
  Arr *v = new_view(a);
  for (int i = 0; i < a->ndim; i++) {
    v->shape[i] = a->shape[perm[i]];
    v->strides[i] = a->strides[perm[i]];
  }
  return v;
}

}  // namespace

struct Tracer {
  int mode = 0;  // 1: logging the eager call, 2: applying the plan in the capture call
  Device *dev = nullptr;
  std::vector<TOp> ops;
  std::vector<uint64_t> outputs;
  std::vector<int> group_of, role_of;
  std::vector<Group> groups;
  size_t next = 0;
  bool diverged = false;
  std::string why;

  ~Tracer() {
    for (Group &g : groups)
      for (Arr *&a : g.h)
        if (a) {
          shlo_release(a);
          a = nullptr;
        }
  }

  void diverge(const char *what) {
    if (!diverged) {
      diverged = true;
      why = what;
    }
  }

  // ---- the plan ----

  void plan() {
    const int n = (int)ops.size();
    std::map<uint64_t, int> uses, user, producer;
    for (int i = 0; i < n; i++) {
      if (ops[i].out) producer[ops[i].out] = i;
      for (const TIn &t : ops[i].in)
        if (t.buf) {
          uses[t.buf]++;
          user[t.buf] = i;
        }
    }
    for (uint64_t o : outputs) uses[o] += 1;
    // the one op that reads `b`, when nothing else does (a function output never qualifies)
    auto single = [&](uint64_t b) -> int {
      auto u = uses.find(b), w = user.find(b);
      return b && u != uses.end() && u->second == 1 && w != user.end() ? w->second : -1;
    };
    auto made_by_copy = [&](uint64_t b) -> int {
      auto it = producer.find(b);
      if (it == producer.end() || ops[it->second].kind != TK_COPY || single(b) < 0) return -1;
      return it->second;
    };
    group_of.assign(n, -1);
    role_of.assign(n, ROLE_NONE);
    auto take = [&](Group &g, std::vector<std::pair<int, int>> members) {
      std::sort(members.begin(), members.end());
      for (auto &m : members)
        if (group_of[m.first] >= 0) return false;
      const int gi = (int)groups.size();
      for (auto &m : members) {
        group_of[m.first] = gi;
        role_of[m.first] = m.second;
        g.ops.push_back(m.first);
        if (m.first > g.last) g.last = m.first;
      }
      groups.push_back(g);
      return true;
    };

    // dense: i is the mul_mat of one weight
    auto try_dense = [&](int i) {
      const TOp &o = ops[i];
      if (o.sub != KK_MUL_MAT || o.p[5] != 0 || o.p[3] != 0 || o.p[4] != o.p[2] || o.in.size() != 3) return;
      const int64_t M = o.p[1], R = o.p[2];
      const int j = single(o.out);
      if (j < 0 || ops[j].kind != TK_BINARY || ops[j].sub != 0 /* add */ || ops[j].in.size() != 2 ||
          ops[j].out_dtype != kF32)
        return;
      const TOp &a = ops[j];
      const int y = full_view(a.in[0], o.out, R * M) ? 0 : full_view(a.in[1], o.out, R * M) ? 1 : -1;
      if (y < 0 || a.out_ndim < 1 || a.out_shape[a.out_ndim - 1] != M) return;
      const TIn &b = a.in[1 - y];
      if (b.buf == o.out || !bcast_last(b, M, a.out_ndim, a.out_shape)) return;
      Group g;
      g.kind = G_DENSE;
      g.flags = EP_BIAS | (y == 1 ? EP_BIAS_LHS : 0);
      for (int k = 0; k < 6; k++) g.p[k] = o.p[k];
      std::vector<std::pair<int, int>> mem = {{i, R_MM}, {j, R_BIAS}};
      uint64_t result = a.out;  // the chain's result so far
      const int k = single(a.out);
      if (k >= 0 && ops[k].kind == TK_BINARY && ops[k].sub == 0 && ops[k].in.size() == 2 && ops[k].out_dtype == kF32) {
        const TOp &r = ops[k];
        const int t = full_view(r.in[0], a.out, R * M) ? 0 : full_view(r.in[1], a.out, R * M) ? 1 : -1;
        if (t >= 0) {
          const TIn &h = r.in[1 - t];
          if (h.buf != a.out && h.dtype == kF32 && row_major(h) && count_of(h) == R * M) {
            g.flags |= EP_RES | (t == 1 ? EP_RES_LHS : 0);
            mem.push_back({k, R_RES});
            result = r.out;
          }
        }
      }
      // then gelu_erf of the whole result (the pinned build's: the stock one is
      // refused, unfused, with its own message)
      const int q = single(result);
      if (q >= 0 && ops[q].kind == TK_KERNEL && ops[q].sub == KK_GELU_ERF && ops[q].np >= 2 &&
          ops[q].p[0] == (uint32_t)(R * M) && ops[q].p[1] == 0 && current_flavor() == 0 && !ops[q].in.empty() &&
          full_view(ops[q].in[0], result, R * M)) {
        g.flags |= EP_GELU;
        mem.push_back({q, R_GELU});
      }
      g.p[6] = (uint32_t)g.flags;
      take(g, mem);
    };

    // attention: i is the scores product, batched over batch and head, K = 64.
    // q, k and v each reach their product either through a copy of a transposed
    // view (the chain's own op) or as a strided view read directly (when the
    // transposed axes merge, e.g. one sample or one head); the chain ends with
    // the copy of the value product into [batch, position, head*64], or at the
    // value product itself when that already is the layout (one head).
    auto try_attention = [&](int i) {
      const TOp &o = ops[i];
      // (Lower.lean gives a product of one batch no weight batch stride)
      if (o.sub != KK_MUL_MAT || o.p[5] != 0 || o.p[0] != 64 || (o.p[1] != 128 && o.p[1] != 256) ||
          o.p[4] != o.p[1] || o.in.size() != 3 || o.p[2] % o.p[1] != 0 ||
          !(o.p[3] == o.p[1] * 64 || (o.p[3] == 0 && o.p[2] == o.p[1])))
        return;
      const int64_t S = o.p[1], R = o.p[2];
      // the batch and head counts, from the copy of q or k (or from the value side below)
      int64_t B = 0, H = 0;
      auto qk_source = [&](const TIn &x, int *copy) -> bool {
        *copy = made_by_copy(x.buf);
        if (*copy >= 0) {
          const TIn &v = ops[*copy].in.size() == 1 ? ops[*copy].in[0] : x;
          if (!full_view(x, x.buf, R * 64) || ops[*copy].in.size() != 1 || v.ndim != 4 || v.dtype != kF32 ||
              v.shape[2] != S || v.shape[3] != 64 || v.shape[0] * v.shape[1] * S != R)
            return false;
          if (B && (v.shape[0] != B || v.shape[1] != H)) return false;
          B = v.shape[0];
          H = v.shape[1];
          return true;
        }
        return x.dtype == kF32 && x.ndim == 2 && x.shape[0] == R && x.shape[1] == 64;  // read directly
      };
      int cq = -1, ck = -1;
      if (!qk_source(o.in[1], &cq) || !qk_source(o.in[0], &ck)) return;
      const int j = single(o.out);
      if (j < 0 || ops[j].kind != TK_KERNEL || ops[j].sub != KK_SOFT_MAX || ops[j].p[0] != S || ops[j].p[1] != R ||
          ops[j].p[3] != 0 || ops[j].in.size() != 2 || !full_view(ops[j].in[0], o.out, R * S))
        return;
      const int l = single(ops[j].out);
      if (l < 0 || ops[l].kind != TK_KERNEL || ops[l].sub != KK_MUL_MAT || ops[l].in.size() != 3) return;
      const TOp &vo = ops[l];
      if (vo.p[0] != S || vo.p[1] != 64 || vo.p[2] != R || vo.p[4] != S || vo.p[5] != 0 ||
          !(vo.p[3] == 64 * S || (vo.p[3] == 0 && R == S)) || !full_view(vo.in[1], ops[j].out, R * S))
        return;
      const TIn &vx = vo.in[0];
      int cv = made_by_copy(vx.buf);
      if (cv >= 0) {
        const TIn &vv = ops[cv].in.size() == 1 ? ops[cv].in[0] : vx;  // [B, H, 64, S]: v transposed
        if (ops[cv].in.size() != 1 || !full_view(vx, vx.buf, R * 64) || vv.ndim != 4 || vv.dtype != kF32 ||
            vv.shape[2] != 64 || vv.shape[3] != S || vv.shape[0] * vv.shape[1] * S != R)
          return;
        if (B && (vv.shape[0] != B || vv.shape[1] != H)) return;
        B = vv.shape[0];
        H = vv.shape[1];
      } else if (!(vx.dtype == kF32 && vx.ndim == 2 && vx.shape[0] == R / S * 64 && vx.shape[1] == S)) {
        return;
      }
      // the end: the copy into [B, S, H*64], or (one head) the value product itself
      int t = single(vo.out);
      if (t >= 0 && ops[t].kind == TK_COPY && ops[t].in.size() == 1) {
        const TIn &ov = ops[t].in[0];  // the value product [B, H, S, 64] read as [B, S, H, 64]
        const int64_t tb = ov.ndim == 4 ? ov.shape[0] : 0, th = ov.ndim == 4 ? ov.shape[2] : 0;
        const int64_t want_st[4] = {th * S * 64, 64, S * 64, 1};
        bool ok = ov.buf == vo.out && ov.offset == 0 && ov.ndim == 4 && ov.dtype == kF32 && tb * th * S == R &&
                  ov.shape[1] == S && ov.shape[3] == 64 && (!B || (tb == B && th == H));
        for (int d = 0; d < 4 && ok; d++) ok = ov.strides[d] == want_st[d] || ov.shape[d] == 1;
        if (ok) {
          B = tb;
          H = th;
        } else {
          t = -1;
        }
      } else {
        t = -1;
      }
      // No copy told the batch from the heads: the products' row blocks are then
      // read as B = batch*head samples of one head, whose output layout is the
      // value product's own.
      if (!B) {
        B = R / S;
        H = 1;
      }
      if (t < 0 && H != 1) return;
      Group g;
      g.kind = G_ATTN;
      g.p[0] = (uint32_t)B;
      g.p[1] = (uint32_t)S;
      g.p[2] = (uint32_t)H;
      g.p[3] = 64;
      g.p[4] = ops[j].p[2];  // soft_max's scale
      std::vector<std::pair<int, int>> mem = {{i, R_SCORES}, {j, R_SOFTMAX}, {l, R_VALUE}};
      if (cq >= 0) mem.push_back({cq, R_CQ});
      if (ck >= 0) mem.push_back({ck, R_CK});
      if (cv >= 0) mem.push_back({cv, R_CV});
      if (t >= 0) mem.push_back({t, R_COPY_OUT});
      g.direct = (cq < 0 ? 1 : 0) | (ck < 0 ? 2 : 0) | (cv < 0 ? 4 : 0);
      take(g, mem);
    };

    // layer norm: i is the norm
    auto try_norm = [&](int i) {
      const TOp &o = ops[i];
      if (o.sub != KK_NORM || o.p[3] != 0 || o.in.size() != 2) return;
      const int64_t C = o.p[0], Rw = o.p[1];
      const int j = single(o.out);
      if (j < 0 || ops[j].kind != TK_BINARY || ops[j].sub != 2 /* mul */ || ops[j].in.size() != 2 ||
          !full_view(ops[j].in[0], o.out, Rw * C) || !bcast_last(ops[j].in[1], C, ops[j].out_ndim, ops[j].out_shape))
        return;
      const int k = single(ops[j].out);
      if (k < 0 || ops[k].kind != TK_BINARY || ops[k].sub != 0 || ops[k].in.size() != 2 ||
          !full_view(ops[k].in[0], ops[j].out, Rw * C) || !bcast_last(ops[k].in[1], C, ops[k].out_ndim, ops[k].out_shape))
        return;
      Group g;
      g.kind = G_NORM;
      for (int q = 0; q < 4; q++) g.p[q] = o.p[q];
      take(g, {{i, R_NORM}, {j, R_GAIN}, {k, R_BETA}});
    };

    for (int i = 0; i < n; i++) {
      if (group_of[i] >= 0 || ops[i].kind != TK_KERNEL) continue;
      try_dense(i);
      if (group_of[i] < 0) try_attention(i);
      if (group_of[i] < 0) try_norm(i);
    }

    // A chain whose result the next dense chain's product alone reads, as its
    // whole x, hands it over packed: dense -> gelu_erf (FFN1 -> FFN2), the
    // attention block (-> the output projection), the layer norm (-> QKV, FFN1).
    for (int a = 0; a < (int)groups.size(); a++) {
      Group &g1 = groups[a];
      int64_t M1, R1;  // the result's row width and rows
      if (g1.kind == G_DENSE && (g1.flags & EP_GELU)) {
        M1 = g1.p[1];
        R1 = g1.p[2];
      } else if (g1.kind == G_ATTN) {
        M1 = (int64_t)g1.p[2] * g1.p[3];
        R1 = (int64_t)g1.p[0] * g1.p[1];
      } else if (g1.kind == G_NORM) {
        M1 = g1.p[0];
        R1 = g1.p[1];
      } else {
        continue;
      }
      const uint64_t r1 = ops[g1.last].out;
      const int j = single(r1);
      if (j < 0 || group_of[j] < 0 || role_of[j] != R_MM) continue;
      Group &g2 = groups[group_of[j]];
      if (g2.kind != G_DENSE || g2.x_np || g2.p[0] != (uint32_t)M1 || g2.p[2] != (uint32_t)R1 ||
          !full_view(ops[j].in[1], r1, R1 * M1) || ops[j].in[0].buf == r1)
        continue;
      int segp, np;
      if (!mm_packed_x_layout(M1, g2.p[1], R1, &segp, &np)) continue;
      g1.y_pack[0] = segp;
      g1.y_pack[1] = np;
      g2.x_np = np;
      g2.src = a;
    }
  }

  // ---- the capture call ----

  // A placeholder result of the logged shape (storage nothing writes or reads).
  int placeholder(const TOp &lo, Group &g, int role, Arr **out) {
    SHLO_TRY(new_array(dev, lo.out_dtype, lo.out_shape, lo.out_ndim, out));
    g.placeholder[role] = (*out)->buf;
    return 0;
  }

  // The chained operand must be a view of the chain's previous placeholder.
  bool chained(Group &g, int role, Arr *a) { return a && a->buf && g.placeholder.count(role) && g.placeholder[role] == a->buf; }

  void set_handle(Group &g, int slot, Arr *v) {
    if (g.h[slot]) shlo_release(g.h[slot]);
    g.h[slot] = v;
  }

  // A [B, S, H, 64] view of a product's 2-D operand read directly: q or k as
  // [B*H*S, 64] rows ((b*H + h)*S + s), or v as [B*H*64, S] rows ((b*H + h)*64 + d).
  static Arr *rows_view(const Arr *a, const uint32_t *p, bool value) {
    const int64_t S = p[1], H = p[2], B = p[0];
    const int64_t rs = a->strides[0], cs = a->strides[1];
    Arr *v = new_view(a);
    v->ndim = 4;
    v->shape[0] = B;
    v->shape[1] = S;
    v->shape[2] = H;
    v->shape[3] = 64;
    if (value) {
      v->strides[0] = H * 64 * rs;
      v->strides[1] = cs;
      v->strides[2] = 64 * rs;
      v->strides[3] = rs;
    } else {
      v->strides[0] = H * S * rs;
      v->strides[1] = rs;
      v->strides[2] = S * rs;
      v->strides[3] = cs;
    }
    return v;
  }

  void keep(Group &g, int slot, Arr *a) {
    a->rc.fetch_add(1);
    if (g.h[slot]) shlo_release(g.h[slot]);
    g.h[slot] = a;
  }

  // The fused launch; *out takes the last op's logged shape.
  int launch(Group &g, const TOp &lo, Arr **out) {
    Arr *o = nullptr;
    Arr *c[4] = {nullptr, nullptr, nullptr, nullptr};
    int rc = 0;
    for (int s = 0; s < 3; s++)  // every kind's first three operands (the residual is optional)
      if (!g.h[s]) return fail("fusion: a chain ended without its operands");
    const int *yp = g.y_pack[1] ? g.y_pack : nullptr;  // the result packed for the next chain
    if (g.kind == G_DENSE) {
      // h: 0 w, 1 x, 2 bias (1-D view), 3 residual
      for (int s = 0; s < 4 && !rc; s++)
        if (g.h[s]) rc = prep(dev, g.h[s], &c[s]);
      if (!rc) rc = k_mul_mat_fused(dev, c[0], c[1], g.p, c[2], c[3], g.flags, g.x_np, yp, &o);
    } else if (g.kind == G_NORM) {
      // h: 0 x, 1 gain (1-D view), 2 bias (1-D view)
      for (int s = 0; s < 3 && !rc; s++) rc = prep(dev, g.h[s], &c[s]);
      if (!rc) rc = k_norm_affine_packed(dev, c[0], g.p, c[1], c[2], yp, &o);
    } else {
      // h: 0 q, 1 k, 2 v, as [B, S, H, 64] views
      rc = k_attention_packed(dev, g.h[0], g.h[1], g.h[2], g.p, yp, &o);
    }
    if (!rc) g.produced = o->buf->serial;
    for (Arr *a : c)
      if (a) shlo_release(a);
    for (Arr *&a : g.h)
      if (a) {
        shlo_release(a);
        a = nullptr;
      }
    if (rc) return 1;
    rc = shlo_reshape(o, lo.out_shape, lo.out_ndim, out);
    shlo_release(o);
    g.done = true;
    return rc;
  }

  // One op of a chain in the capture call. Returns 0 with *out set, or 1 on error.
  int apply(int idx, Arr *const *ins, int n, Arr **out) {
    Group &g = groups[group_of[idx]];
    const TOp &lo = ops[idx];
    const int role = role_of[idx];
    bool ok = true;
    if (g.kind == G_DENSE) {
      if (role == R_MM) {
        // a packed x must be the linked chain's fused result itself
        ok = !g.x_np || (ins[1]->buf && groups[g.src].done && ins[1]->buf->serial == groups[g.src].produced &&
                         ins[1]->offset == 0);
        keep(g, 0, ins[0]);
        keep(g, 1, ins[1]);
      } else if (role == R_BIAS) {
        const int y = chained(g, R_MM, ins[0]) ? 0 : chained(g, R_MM, ins[1]) ? 1 : -1;
        ok = y >= 0 && ((g.flags & EP_BIAS_LHS) != 0) == (y == 1);
        if (ok) {
          Arr *b = new_view(ins[1 - y]);  // the bias as its 1-D vector
          b->ndim = 1;
          b->shape[0] = ins[1 - y]->shape[ins[1 - y]->ndim - 1];
          b->strides[0] = 1;
          if (g.h[2]) shlo_release(g.h[2]);
          g.h[2] = b;
        }
      } else if (role == R_RES) {
        const int t = chained(g, R_BIAS, ins[0]) ? 0 : chained(g, R_BIAS, ins[1]) ? 1 : -1;
        ok = t >= 0 && ((g.flags & EP_RES_LHS) != 0) == (t == 1);
        if (ok) keep(g, 3, ins[1 - t]);
      } else {  // gelu_erf of the chain's result
        ok = n >= 1 && chained(g, (g.flags & EP_RES) ? R_RES : R_BIAS, ins[0]);
      }
    } else if (g.kind == G_NORM) {
      if (role == R_NORM) {
        keep(g, 0, ins[0]);
      } else {
        ok = chained(g, role == R_GAIN ? R_NORM : R_GAIN, ins[0]);
        if (ok) {
          Arr *v = new_view(ins[1]);
          v->ndim = 1;
          v->shape[0] = ins[1]->shape[ins[1]->ndim - 1];
          v->strides[0] = 1;
          if (g.h[role == R_GAIN ? 1 : 2]) shlo_release(g.h[role == R_GAIN ? 1 : 2]);
          g.h[role == R_GAIN ? 1 : 2] = v;
        }
      }
    } else {
      static const int to_bshd[4] = {0, 2, 1, 3};  // [B, H, S, 64] -> [B, S, H, 64]
      static const int v_to_bshd[4] = {0, 3, 1, 2};  // [B, H, 64, S] -> [B, S, H, 64]
      switch (role) {
        case R_CQ:
        case R_CK: {
          Arr *v = permuted(ins[0], to_bshd);
          if (g.h[role == R_CQ ? 0 : 1]) shlo_release(g.h[role == R_CQ ? 0 : 1]);
          g.h[role == R_CQ ? 0 : 1] = v;
          break;
        }
        case R_CV: {
          Arr *v = permuted(ins[0], v_to_bshd);
          if (g.h[2]) shlo_release(g.h[2]);
          g.h[2] = v;
          break;
        }
        case R_SCORES:
          ok = ((g.direct & 2) || chained(g, R_CK, ins[0])) && ((g.direct & 1) || chained(g, R_CQ, ins[1]));
          if (ok && (g.direct & 1)) set_handle(g, 0, rows_view(ins[1], g.p, false));
          if (ok && (g.direct & 2)) set_handle(g, 1, rows_view(ins[0], g.p, false));
          break;
        case R_SOFTMAX: ok = chained(g, R_SCORES, ins[0]); break;
        case R_VALUE:
          ok = ((g.direct & 4) || chained(g, R_CV, ins[0])) && chained(g, R_SOFTMAX, ins[1]);
          if (ok && (g.direct & 4)) set_handle(g, 2, rows_view(ins[0], g.p, true));
          break;
        case R_COPY_OUT: ok = chained(g, R_VALUE, ins[0]); break;
      }
    }
    (void)n;
    if (!ok) {
      diverge("a fused chain's operands differ from the eager call's");
      return -1;
    }
    if (idx == g.last) return launch(g, lo, out);
    return placeholder(lo, g, role, out);
  }

  bool complete() const {
    if (diverged || next != ops.size()) return false;
    for (const Group &g : groups)
      if (!g.done) return false;
    return true;
  }
};

bool fusion_enabled() {
  static const bool on = [] {
    const char *e = getenv("SHLO_FUSE");
    return !(e && strcmp(e, "0") == 0);
  }();
  return on;
}

Tracer *tracer_new(Device *dev) {
  Tracer *t = new Tracer();
  t->mode = 1;
  t->dev = dev;
  return t;
}

void tracer_free(Tracer *t) { delete t; }

// $SHLO_GRAPH_VERBOSE=2: the op log of each recording and the chains found in it.
static void dump_log(const Tracer *t) {
  static const char *kinds[] = {"?", "kernel", "binary", "copy", "other"};
  for (size_t i = 0; i < t->ops.size(); i++) {
    const TOp &o = t->ops[i];
    fprintf(stderr, "shlo log %zu: %s %d p=[", i, kinds[o.kind < 5 ? o.kind : 0], o.sub);
    for (int k = 0; k < o.np; k++) fprintf(stderr, "%s%u", k ? "," : "", o.p[k]);
    fprintf(stderr, "] ->#%llu chain %d role %d\n", (unsigned long long)o.out, t->group_of[i], t->role_of[i]);
    for (const TIn &x : o.in) {
      fprintf(stderr, "    in #%llu dt %d off %lld shape", (unsigned long long)x.buf, (int)x.dtype, (long long)x.offset);
      for (int d = 0; d < x.ndim; d++) fprintf(stderr, " %lld:%lld", (long long)x.shape[d], (long long)x.strides[d]);
      fprintf(stderr, "\n");
    }
  }
}

int tracer_plan(Tracer *t, Arr *const *outs, int n) {
  for (int i = 0; i < n; i++)
    if (outs[i] && outs[i]->buf) t->outputs.push_back(outs[i]->buf->serial);
  t->plan();
  const char *v = getenv("SHLO_GRAPH_VERBOSE");
  if (v && atoi(v) >= 2) dump_log(t);
  if (v && atoi(v) >= 1) {
    int links = 0;
    for (const Group &g : t->groups) links += g.y_pack[1] != 0;
    if (links) fprintf(stderr, "shlo: fused chains handing a packed operand on: %d\n", links);
  }
  t->mode = 2;
  t->next = 0;
  return (int)t->groups.size();
}

bool tracer_complete(Tracer *t, std::string *why) {
  if (t->complete()) return true;
  *why = t->diverged ? t->why : "the capture call did not reach every fused chain's end";
  return false;
}

// ---- TraceScope ----

TraceScope::TraceScope(int kind, int sub, const uint32_t *p, int np, Arr *const *ins, int n) {
  depth_ = ++t_trace_depth;
  Tracer *t = t_tracer;
  if (!t || depth_ != 1 || kind == 0) return;  // kind 0: this call reads no data
  if (t->mode == 1) {
    idx_ = (int)t->ops.size();
    TOp o;
    o.kind = kind;
    o.sub = sub;
    o.np = np < 8 ? np : 8;
    for (int k = 0; k < o.np; k++) o.p[k] = p[k];
    for (int k = 0; k < n; k++)
      if (ins[k]) o.in.push_back(in_of(ins[k]));
    t->ops.push_back(o);
    logging_ = true;
    return;
  }
  // the capture call
  const size_t idx = t->next++;
  if (t->diverged) return;
  if (idx >= t->ops.size()) {
    t->diverge("the capture call has more ops than the eager call");
    return;
  }
  const TOp &lo = t->ops[idx];
  bool same = lo.kind == kind && lo.sub == sub && (int)lo.in.size() <= n;
  for (int k = 0; k < lo.np && same; k++) same = k < np && lo.p[k] == p[k];
  int m = 0;
  for (int k = 0; k < n && same; k++)
    if (ins[k]) same = m < (int)lo.in.size() && same_layout(lo.in[m++], in_of(ins[k]));
  if (!same || m != (int)lo.in.size()) {
    t->diverge("the capture call's ops differ from the eager call's");
    return;
  }
  if (t->group_of[idx] < 0) return;
  Arr *r = nullptr;
  const int rc = t->apply((int)idx, ins, n, &r);
  if (rc < 0) return;  // diverged: the op runs as it is
  substituted_ = true;
  status_ = rc;
  result_ = r;
}

TraceScope::~TraceScope() { t_trace_depth--; }

void TraceScope::done(Arr *out) {
  if (!logging_) return;
  Tracer *t = t_tracer;
  if (!t || t->mode != 1 || idx_ < 0 || idx_ >= (int)t->ops.size()) return;
  TOp &o = t->ops[idx_];
  if (out && out->buf) {
    o.out = out->buf->serial;
    o.out_dtype = out->dtype;
    o.out_ndim = out->ndim;
    for (int i = 0; i < out->ndim; i++) o.out_shape[i] = out->shape[i];
  }
}

}  // namespace shlo
