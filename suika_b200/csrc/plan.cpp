// Transfer planner of the B200 live-reshard path (host C++17, C ABI in include/suika_reshard.h).
//
// rs_plan_build restates Suika's schedule_param_transfer (Suika/migration.py:322-381) over flat
// descriptors: the same target iteration order, the same rescale of every target tensor to the
// largest source TP degree (TensorMeta.scale_to_tp, migration.py:103-118), the same ownership
// test (ParamLayout.is_tensor_tp_owned / is_tensor_tp_overlap, migration.py:220-254) and the same
// greedy source choice (migration.py:355-379), so the op list equals the reference's op for op.
//
// rs_program_build turns the ops whose target is one rank into in-place strided copies: the
// reference's get_send_tensor chunk + contiguous (migration.py:290-312), the per-tensor
// isend/irecv (migration.py:466,489) and the final torch.cat / clone (migration.py:531-545)
// collapse into one (rows x row_bytes, pitch) copy per piece and sub-field, written straight
// into its final position of the target tensor.
#include "../../include/suika_reshard.h"
#include "internal.h"

#include <algorithm>
#include <cstring>
#include <map>
#include <tuple>
#include <new>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) { return suika_rs::fail(code, msg); }

// Records msg (which may describe objects owned by p) and only then frees p.
template <class T>
int fail_and_free(T* p, int code, const std::string& msg) {
  const int rc = suika_rs::fail(code, msg);
  delete p;
  return rc;
}

struct Meta {
  int32_t name = -1;
  int32_t ndim = 0;
  int64_t shape[RS_MAX_DIMS] = {0};
  int32_t itemsize = 0;
  int32_t slice_dim = RS_NO_SLICE;
  int32_t tp_index = 0;
  int32_t tp_deg = 1;

  bool is_tp() const { return slice_dim != RS_NO_SLICE; }
  int32_t deg() const { return is_tp() ? tp_deg : 1; }
  int32_t idx() const { return is_tp() ? tp_index : 0; }
  int64_t full_numel() const {
    int64_t n = 1;
    for (int i = 0; i < ndim; ++i) n *= shape[i];
    return n;
  }
  // TensorMeta.numel(): prod(shape) // tp_deg (migration.py:66-67).
  int64_t numel() const { return full_numel() / deg(); }
  // TensorMeta.volumn(): numel * itemsize (migration.py:70-71).
  int64_t volume() const { return numel() * itemsize; }
  int norm_dim() const { return slice_dim < 0 ? slice_dim + ndim : slice_dim; }
};

struct RankLayout {
  int32_t rank = 0;
  std::vector<Meta> tensors;
  std::unordered_map<int32_t, int32_t> by_name;  // name -> index in tensors
};

std::string meta_str(const Meta& m) {
  std::string s = "(name_id=" + std::to_string(m.name) + ", shape=[";
  for (int i = 0; i < m.ndim; ++i) s += (i ? "," : "") + std::to_string(m.shape[i]);
  s += "], tp=";
  if (m.is_tp())
    s += "(" + std::to_string(m.slice_dim) + "," + std::to_string(m.tp_index) + "," + std::to_string(m.tp_deg) + ")";
  else
    s += "None";
  return s + ")";
}

int load_layout(const rs_rank_layout* in, int32_t n, std::vector<RankLayout>& out, const char* what) {
  if (n < 0 || (n > 0 && !in)) return fail(RS_ERR_ARG, std::string(what) + ": bad layout array");
  out.resize(n);
  std::unordered_set<int32_t> ranks;
  for (int32_t r = 0; r < n; ++r) {
    RankLayout& L = out[r];
    L.rank = in[r].rank;
    if (!ranks.insert(L.rank).second)
      return fail(RS_ERR_ARG, std::string(what) + ": rank " + std::to_string(L.rank) + " listed twice");
    if (in[r].n_tensors < 0 || (in[r].n_tensors > 0 && !in[r].tensors))
      return fail(RS_ERR_ARG, std::string(what) + ": bad tensor array for rank " + std::to_string(L.rank));
    L.tensors.resize(in[r].n_tensors);
    for (int32_t t = 0; t < in[r].n_tensors; ++t) {
      const rs_tensor_meta& s = in[r].tensors[t];
      Meta& m = L.tensors[t];
      m.name = s.name_id;
      m.ndim = s.ndim;
      m.itemsize = s.itemsize;
      m.slice_dim = s.slice_dim;
      m.tp_index = s.tp_index;
      m.tp_deg = s.tp_deg;
      if (s.ndim < 0 || s.ndim > RS_MAX_DIMS || s.itemsize <= 0 || s.name_id < 0)
        return fail(RS_ERR_ARG, std::string(what) + ": malformed tensor meta on rank " + std::to_string(L.rank));
      for (int i = 0; i < s.ndim; ++i) {
        if (s.shape[i] < 0) return fail(RS_ERR_ARG, std::string(what) + ": negative dim");
        m.shape[i] = s.shape[i];
      }
      if (m.is_tp()) {
        if (s.tp_deg < 1 || s.tp_index < 0 || s.tp_index >= s.tp_deg || s.slice_dim < -s.ndim || s.slice_dim >= s.ndim)
          return fail(RS_ERR_ARG, std::string(what) + ": malformed tp_meta " + meta_str(m) + " on rank " + std::to_string(L.rank));
      }
      if (!L.by_name.emplace(m.name, t).second)
        return fail(RS_ERR_ARG, std::string(what) + ": name_id " + std::to_string(m.name) + " twice on rank " + std::to_string(L.rank));
    }
  }
  return RS_OK;
}

// ParamLayout.is_tensor_tp_overlap (migration.py:220-244). Returns -1 on the reference's
// slice-dim assertion.
int tp_overlap(const Meta& a, const Meta& b) {
  if (!a.is_tp() || !b.is_tp()) return 1;
  if (a.slice_dim != b.slice_dim) return -1;
  int64_t i1 = a.tp_index, g1 = a.tp_deg, i2 = b.tp_index, g2 = b.tp_deg;
  if (g1 > g2) {
    std::swap(i1, i2);
    std::swap(g1, g2);
  }
  const int64_t scale = g2 / g1;
  return (i2 / scale == i1) ? 1 : 0;
}

// ParamLayout.is_tensor_tp_owned (migration.py:246-254).
int tp_owned(const Meta& src, const Meta& tgt) {
  if (!(src.deg() <= tgt.deg())) return 0;
  return tp_overlap(src, tgt);
}

}  // namespace

int suika_rs::fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

// A piece of the interval planner, in units of the slice dim: `len` indices starting at
// src_start of the source shard's storage go to dst_start of the target shard's storage. Whole
// (unsliced) tensors use outer = 1, inner = numel, extents = len = 1.
struct Piece {
  int32_t name = -1, src_rank = -1, dst_rank = -1;
  int64_t outer = 1, inner = 1;
  int64_t src_extent = 1, dst_extent = 1;
  int64_t src_start = 0, dst_start = 0, len = 1;
  int64_t src_numel = 0;          // elements of the source shard
  int32_t ndim = 0;
  int64_t dst_shape[RS_MAX_DIMS] = {0};  // actual shape of the target shard
};

struct Rule {
  int32_t n_groups = 0;
  rs_slice_group groups[RS_MAX_GROUPS];
};

struct rs_plan {
  int32_t mode = 0;  // 0: reference schedule (rs_plan_build), 1: interval intersection (rs_plan_build_rules)
  std::vector<Piece> pieces;  // mode 1: per target rank, target tensor order, storage order
  std::vector<RankLayout> src, dst;
  std::vector<rs_op> ops;
  std::vector<Meta> src_meta_of_op;  // src meta per op
  std::vector<Meta> dst_meta_of_op;  // rescaled target piece per op
  std::vector<Meta> dst_full_of_op;  // the target rank's own meta (unscaled)
  int32_t order = RS_ORDER_REFERENCE;
  int32_t max_tp = 1;
};

extern "C" {

const char* rs_last_error(void) { return g_err.c_str(); }

// schedule_param_transfer, Suika/migration.py:322-381.
int rs_plan_build(const rs_rank_layout* src, int32_t n_src, const rs_rank_layout* dst, int32_t n_dst,
                  const rs_plan_opts* opts, rs_plan** out) {
  if (!out) return fail(RS_ERR_ARG, "rs_plan_build: out is NULL");
  *out = nullptr;
  rs_plan* plan = new (std::nothrow) rs_plan();
  if (!plan) return fail(RS_ERR_ARG, "rs_plan_build: out of host memory");
  try {
    int rc = load_layout(src, n_src, plan->src, "source layout");
    if (rc) { delete plan; return rc; }
    rc = load_layout(dst, n_dst, plan->dst, "target layout");
    if (rc) { delete plan; return rc; }
    const int32_t min_est = opts ? opts->minimum_est_peers : 2;
    const int32_t choice = opts ? opts->src_choice : RS_SRC_REFERENCE;
    plan->order = opts ? opts->order : RS_ORDER_REFERENCE;
    if (plan->order != RS_ORDER_REFERENCE && plan->order != RS_ORDER_SEMANTIC) {
      return fail_and_free(plan, RS_ERR_ARG, "rs_plan_build: unknown order");
    }

    // max_tp_degree over every source tensor (migration.py:335); max() of nothing raises.
    bool any = false;
    int32_t max_tp = 1;
    for (const RankLayout& L : plan->src)
      for (const Meta& m : L.tensors) {
        max_tp = any ? std::max(max_tp, m.deg()) : m.deg();
        any = true;
      }
    if (!any) {
      return fail_and_free(plan, RS_ERR_EMPTY_SOURCE, "schedule_param_transfer: source layout holds no tensor (max() arg is an empty sequence)");
    }
    plan->max_tp = max_tp;

    // latency_vec = [0.0 for rank in spl.layout.keys()], indexed by rank value (migration.py:339).
    std::vector<double> latency(plan->src.size(), 0.0);
    for (const RankLayout& L : plan->src)
      if (L.rank < 0 || L.rank >= (int32_t)plan->src.size()) {
        return fail_and_free(plan, RS_ERR_ARG, "schedule_param_transfer: source rank " + std::to_string(L.rank) +
                                    " outside range(len(spl.layout)) (latency_vec index)");
      }

    std::vector<int32_t> owners;
    std::vector<char> est(plan->src.size(), 0);
    std::vector<size_t> deferred;                     // ops whose source the balanced rule picks
    std::vector<std::vector<int32_t>> deferred_owners;
    auto set_source = [&](size_t i, int32_t best) {
      const RankLayout* S = nullptr;
      for (const RankLayout& L : plan->src)
        if (L.rank == best) { S = &L; break; }
      const Meta& sm = S->tensors[S->by_name.at(plan->ops[i].name_id)];
      rs_op& op = plan->ops[i];
      op.src_rank = best;
      op.src_slice_dim = sm.slice_dim;
      op.src_tp_index = sm.is_tp() ? sm.tp_index : 0;
      op.src_tp_deg = sm.is_tp() ? sm.tp_deg : 1;
      plan->src_meta_of_op[i] = sm;
    };
    for (const RankLayout& D : plan->dst) {
      std::fill(est.begin(), est.end(), 0);  // est_peers = set() per target rank (migration.py:346)
      int32_t n_est = 0;
      for (const Meta& orig : D.tensors) {
        // scale_to_tp(max_tp_degree) (migration.py:103-118, called at :351).
        std::vector<Meta> pieces;
        if (orig.is_tp() && max_tp > orig.tp_deg) {
          const int32_t scale = max_tp / orig.tp_deg;
          for (int32_t i = 0; i < scale; ++i) {
            Meta p = orig;
            p.tp_index = scale * orig.tp_index + i;
            p.tp_deg = max_tp;
            pieces.push_back(p);
          }
        } else {
          pieces.push_back(orig);
        }
        for (const Meta& piece : pieces) {
          // srcs = spl.owners(dst_param) (migration.py:354, 207-208), in layout order.
          owners.clear();
          bool self_owned = false;
          for (const RankLayout& S : plan->src) {
            auto it = S.by_name.find(piece.name);
            if (it == S.by_name.end()) continue;
            const int o = tp_owned(S.tensors[it->second], piece);
            if (o < 0) {
              return fail_and_free(plan, RS_ERR_SLICE_DIM, "slice dim mismatch between " + meta_str(S.tensors[it->second]) + " and " + meta_str(piece));
            }
            if (o) {
              owners.push_back(S.rank);
              if (S.rank == D.rank) self_owned = true;
            }
          }
          if (owners.empty()) {
            return fail_and_free(plan, RS_ERR_NO_OWNER, "illegal transfer, target param " + meta_str(piece) + " of rank " + std::to_string(D.rank) +
                                             " is not present in any source");
          }
          const double vol = (double)piece.volume();
          int32_t best = -1;
          if (self_owned) {
            best = D.rank;  // migration.py:358-359
          } else if (choice == RS_SRC_BALANCED) {
            deferred.push_back(plan->ops.size());  // chosen after all pieces are known (below)
            deferred_owners.push_back(owners);
          } else {
            // est_srcs first once enough peers are established (migration.py:362-367); min() keeps the first minimum.
            bool use_est = false;
            if (n_est >= min_est)
              for (int32_t s : owners)
                if (est[s]) { use_est = true; break; }
            double best_key = 0.0;
            for (int32_t s : owners) {
              if (use_est && !est[s]) continue;
              const double key = latency[s] + vol;
              if (best < 0 || key < best_key) { best = s; best_key = key; }
            }
          }
          rs_op op;
          std::memset(&op, 0, sizeof(op));
          op.name_id = piece.name;
          op.src_rank = best;
          op.dst_rank = D.rank;
          op.dst_slice_dim = piece.slice_dim;
          op.dst_tp_index = piece.is_tp() ? piece.tp_index : 0;
          op.dst_tp_deg = piece.is_tp() ? piece.tp_deg : 1;
          op.numel = piece.numel();
          plan->ops.push_back(op);
          plan->src_meta_of_op.push_back(Meta());
          plan->dst_meta_of_op.push_back(piece);
          plan->dst_full_of_op.push_back(orig);
          if (best >= 0) {
            if (!est[best]) { est[best] = 1; ++n_est; }
            set_source(plan->ops.size() - 1, best);
            latency[best] += vol;  // migration.py:379
          }
        }
      }
    }
    // Balanced choice: largest pieces first, each to the owner with the least egress so far
    // (ties: first owner in layout order). Op order stays the reference's.
    if (!deferred.empty()) {
      std::vector<size_t> by_size(deferred.size());
      for (size_t i = 0; i < by_size.size(); ++i) by_size[i] = i;
      std::stable_sort(by_size.begin(), by_size.end(), [&](size_t a, size_t b) {
        return plan->dst_meta_of_op[deferred[a]].volume() > plan->dst_meta_of_op[deferred[b]].volume();
      });
      for (size_t k : by_size) {
        const size_t i = deferred[k];
        int32_t best = -1;
        for (int32_t s : deferred_owners[k])
          if (best < 0 || latency[s] < latency[best]) best = s;
        set_source(i, best);
        latency[best] += (double)plan->dst_meta_of_op[i].volume();
      }
    }
  } catch (const std::exception& e) {
    return fail_and_free(plan, RS_ERR_ARG, std::string("rs_plan_build: ") + e.what());
  }
  *out = plan;
  return RS_OK;
}

int rs_plan_num_ops(const rs_plan* plan, int64_t* n_ops) {
  if (!plan || !n_ops) return fail(RS_ERR_ARG, "rs_plan_num_ops: NULL argument");
  *n_ops = (int64_t)plan->ops.size();
  return RS_OK;
}

int rs_plan_get_ops(const rs_plan* plan, rs_op* ops, int64_t capacity) {
  if (!plan || (!ops && !plan->ops.empty())) return fail(RS_ERR_ARG, "rs_plan_get_ops: NULL argument");
  if (capacity < (int64_t)plan->ops.size()) return fail(RS_ERR_CAPACITY, "rs_plan_get_ops: capacity too small");
  if (!plan->ops.empty()) std::memcpy(ops, plan->ops.data(), plan->ops.size() * sizeof(rs_op));
  return RS_OK;
}

void rs_plan_free(rs_plan* plan) { delete plan; }

int rs_version(int32_t* major, int32_t* minor) {
  if (major) *major = 1;
  if (minor) *minor = 2;
  return RS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Per-rank program (execute_param_transfer, Suika/migration.py:397-556, for the ops whose
// target is `rank`).
// ---------------------------------------------------------------------------------------------
struct rs_program {
  int32_t rank = -1;
  std::vector<rs_dst_slot> dst;
  std::vector<rs_src_slot> src;
  std::vector<rs_meta_slot> meta;
  std::vector<rs_segment> segs;
  uint64_t remote_bytes = 0, local_bytes = 0;
};

namespace {

struct PieceGeom {
  // A piece in element units along the normalized slice dim: outer rows x (extent * inner).
  int64_t outer = 1, inner = 1;   // products of dims before / after the slice dim
  int64_t src_extent = 0;         // slice-dim extent of the source tensor
  int64_t piece_extent = 0;       // slice-dim extent of the piece
  int64_t src_start = 0;          // piece start inside the source tensor, along the slice dim
  bool whole = false;             // the piece is the whole source tensor (1 contiguous run)
  int64_t numel = 0;
};

// get_send_tensor (migration.py:290-312) as geometry: returns RS_OK and fills g, or an error.
int piece_geometry(const Meta& sm, const Meta& piece, PieceGeom& g) {
  if (sm.ndim != piece.ndim) return fail(RS_ERR_SHAPE, "rank mismatch between source " + meta_str(sm) + " and target " + meta_str(piece));
  for (int i = 0; i < sm.ndim; ++i)
    if (sm.shape[i] != piece.shape[i])
      return fail(RS_ERR_SHAPE, "full shape mismatch between source " + meta_str(sm) + " and target " + meta_str(piece));
  // assert src_meta.slice_dim() == dst_meta.slice_dim() (migration.py:294).
  if (sm.is_tp() != piece.is_tp() || (sm.is_tp() && sm.slice_dim != piece.slice_dim))
    return fail(RS_ERR_SLICE_DIM, "get_send_tensor: slice dim mismatch btw src " + meta_str(sm) + " and dst " + meta_str(piece));
  if (!sm.is_tp()) {
    g.whole = true;
    g.numel = sm.full_numel();
    return RS_OK;
  }
  const int d = sm.norm_dim();
  const int64_t F = sm.shape[d];
  if (F % sm.tp_deg != 0 || F % piece.tp_deg != 0)
    return fail(RS_ERR_SHAPE, "slice dim extent not divisible by tp degree: " + meta_str(sm) + " / " + meta_str(piece));
  for (int i = 0; i < d; ++i) g.outer *= sm.shape[i];
  for (int i = d + 1; i < sm.ndim; ++i) g.inner *= sm.shape[i];
  g.src_extent = F / sm.tp_deg;
  g.piece_extent = F / piece.tp_deg;
  if (sm.tp_deg >= piece.tp_deg) {  // case 1: send the entire source tensor
    if (g.src_extent != g.piece_extent)
      return fail(RS_ERR_SHAPE, "send tensor shape mismatch: " + meta_str(sm) + " vs " + meta_str(piece));
    g.whole = true;
  } else {  // case 2: chunk(dst_deg // src_deg, dim)[dst_idx - src_idx * chunk_num]
    const int64_t k = piece.tp_deg / sm.tp_deg;
    const int64_t j = (int64_t)piece.tp_index - (int64_t)sm.tp_index * k;
    if (piece.tp_deg % sm.tp_deg != 0 || j < 0 || j >= k)
      return fail(RS_ERR_SHAPE, "get_send_tensor: chunk of " + meta_str(sm) + " does not match " + meta_str(piece));
    g.src_start = j * g.piece_extent;
  }
  g.numel = g.outer * g.piece_extent * g.inner;
  return RS_OK;
}

template <class T>
int copy_out(const std::vector<T>& v, T* out, int64_t capacity, const char* fn) {
  if (!out && !v.empty()) return fail(RS_ERR_ARG, std::string(fn) + ": NULL output");
  if (capacity < (int64_t)v.size()) return fail(RS_ERR_CAPACITY, std::string(fn) + ": capacity too small");
  if (!v.empty()) std::memcpy(out, v.data(), v.size() * sizeof(T));
  return RS_OK;
}

// Program of a plan made by rs_plan_build_rules: the pieces of `rank`, already in target storage
// order, become one segment per piece and sub-field.
int program_from_pieces(const rs_plan* plan, int32_t rank, const rs_subfield* subfields, int32_t n_subfields,
                        rs_program* prog) {
  std::map<std::tuple<int32_t, int32_t, int32_t>, int32_t> src_slot_of;
  size_t i = 0;
  const size_t n = plan->pieces.size();
  while (i < n) {
    if (plan->pieces[i].dst_rank != rank) { ++i; continue; }
    size_t j = i;
    while (j < n && plan->pieces[j].dst_rank == rank && plan->pieces[j].name == plan->pieces[i].name) ++j;
    const Piece& first = plan->pieces[i];
    int64_t numel = 1;
    for (int k = 0; k < first.ndim; ++k) numel *= first.dst_shape[k];
    for (int32_t f = 0; f < n_subfields; ++f) {
      const int64_t E = subfields[f].itemsize;
      if (subfields[f].is_meta) {
        rs_meta_slot ms;
        ms.name_id = first.name;
        ms.subfield = f;
        ms.src_rank = first.src_rank;
        ms.first_is_self = first.src_rank == rank ? 1 : 0;
        prog->meta.push_back(ms);
        continue;
      }
      rs_dst_slot ds;
      std::memset(&ds, 0, sizeof(ds));
      ds.name_id = first.name;
      ds.subfield = f;
      ds.ndim = first.ndim;
      for (int k = 0; k < first.ndim; ++k) ds.shape[k] = first.dst_shape[k];
      ds.nbytes = (uint64_t)(numel * E);
      const int32_t dslot = (int32_t)prog->dst.size();
      prog->dst.push_back(ds);
      for (size_t q = i; q < j; ++q) {
        const Piece& pc = plan->pieces[q];
        auto key = std::make_tuple(pc.src_rank, pc.name, f);
        auto it = src_slot_of.find(key);
        int32_t sslot;
        if (it == src_slot_of.end()) {
          rs_src_slot ss;
          std::memset(&ss, 0, sizeof(ss));
          ss.src_rank = pc.src_rank;
          ss.name_id = pc.name;
          ss.subfield = f;
          ss.nbytes = (uint64_t)(pc.src_numel * E);
          sslot = (int32_t)prog->src.size();
          prog->src.push_back(ss);
          src_slot_of.emplace(key, sslot);
        } else {
          sslot = it->second;
        }
        rs_segment sg;
        std::memset(&sg, 0, sizeof(sg));
        sg.src_slot = sslot;
        sg.dst_slot = dslot;
        sg.rows = (uint64_t)pc.outer;
        sg.row_bytes = (uint64_t)(pc.len * pc.inner * E);
        sg.src_pitch = (uint64_t)(pc.src_extent * pc.inner * E);
        sg.dst_pitch = (uint64_t)(pc.dst_extent * pc.inner * E);
        sg.src_offset = (uint64_t)(pc.src_start * pc.inner * E);
        sg.dst_offset = (uint64_t)(pc.dst_start * pc.inner * E);
        if (sg.rows == 1 || (sg.src_pitch == sg.row_bytes && sg.dst_pitch == sg.row_bytes)) {
          sg.row_bytes *= sg.rows;
          sg.rows = 1;
          sg.src_pitch = sg.dst_pitch = sg.row_bytes;
        }
        const uint64_t bytes = sg.rows * sg.row_bytes;
        if (pc.src_rank == rank) prog->local_bytes += bytes; else prog->remote_bytes += bytes;
        if (bytes > 0) prog->segs.push_back(sg);
      }
    }
    i = j;
  }
  return RS_OK;
}

}  // namespace

extern "C" {

int rs_program_build(const rs_plan* plan, int32_t rank, const rs_subfield* subfields, int32_t n_subfields,
                     rs_program** out) {
  if (!plan || !out || n_subfields < 0 || (n_subfields > 0 && !subfields))
    return fail(RS_ERR_ARG, "rs_program_build: bad argument");
  *out = nullptr;
  for (int32_t f = 0; f < n_subfields; ++f)
    if (subfields[f].itemsize <= 0) return fail(RS_ERR_SUBFIELD, "rs_program_build: sub-field itemsize must be positive");
  rs_program* prog = new (std::nothrow) rs_program();
  if (!prog) return fail(RS_ERR_ARG, "rs_program_build: out of host memory");
  prog->rank = rank;
  try {
    if (plan->mode == 1) {
      int rc = program_from_pieces(plan, rank, subfields, n_subfields, prog);
      if (rc) {
        delete prog;
        return rc;
      }
      *out = prog;
      return RS_OK;
    }
    // Group this rank's ops by target tensor, tensors in first-op order (the creation order of
    // target_state_dict entries, migration.py:431-433).
    std::vector<int32_t> names;
    std::unordered_map<int32_t, std::vector<size_t>> ops_of;
    for (size_t i = 0; i < plan->ops.size(); ++i) {
      const rs_op& op = plan->ops[i];
      if (op.dst_rank != rank) continue;
      auto it = ops_of.find(op.name_id);
      if (it == ops_of.end()) {
        names.push_back(op.name_id);
        ops_of[op.name_id].push_back(i);
      } else {
        it->second.push_back(i);
      }
    }
    std::map<std::tuple<int32_t, int32_t, int32_t>, int32_t> src_slot_of;  // (src rank, name, field)
    for (int32_t name : names) {
      const std::vector<size_t>& idx = ops_of[name];
      // Cat order of the pieces. Reference: received pieces are appended while the ops are
      // issued, self pieces by deferred closures after all issues (migration.py:448-459, 472-492,
      // 508-509), so remote pieces come first. Semantic: slice order.
      std::vector<size_t> order;
      if (plan->order == RS_ORDER_REFERENCE) {
        for (size_t i : idx) if (plan->ops[i].src_rank != rank) order.push_back(i);
        for (size_t i : idx) if (plan->ops[i].src_rank == rank) order.push_back(i);
      } else {
        order = idx;
        std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) {
          return plan->dst_meta_of_op[a].idx() < plan->dst_meta_of_op[b].idx();
        });
      }
      const Meta& full = plan->dst_full_of_op[idx[0]];
      std::vector<PieceGeom> geo(order.size());
      int64_t total_extent = 0;
      for (size_t p = 0; p < order.size(); ++p) {
        const size_t i = order[p];
        int rc = piece_geometry(plan->src_meta_of_op[i], plan->dst_meta_of_op[i], geo[p]);
        if (rc) {
          delete prog;
          return rc;
        }
        total_extent += geo[p].piece_extent;
      }
      // Target tensor shape: pieces concatenated along the slice dim (or the single piece).
      int64_t shape[RS_MAX_DIMS] = {0};
      for (int k = 0; k < full.ndim; ++k) shape[k] = full.shape[k];
      const bool tp = plan->dst_meta_of_op[order[0]].is_tp();
      int d = 0;
      if (tp) {
        d = plan->dst_meta_of_op[order[0]].norm_dim();
        shape[d] = total_extent;
        if (full.is_tp() && full.norm_dim() == d && full.shape[d] % full.tp_deg == 0 && total_extent != full.shape[d] / full.tp_deg) {
          return fail_and_free(prog, RS_ERR_SHAPE, "pieces of " + meta_str(full) + " do not tile its shard");
        }
      } else if (order.size() != 1) {
        return fail_and_free(prog, RS_ERR_SHAPE, "replicated tensor " + meta_str(full) + " built from several pieces");
      }
      int64_t numel = 1;
      for (int k = 0; k < full.ndim; ++k) numel *= shape[k];

      for (int32_t f = 0; f < n_subfields; ++f) {
        const int64_t E = subfields[f].itemsize;
        if (subfields[f].is_meta) {
          // tensors[0].clone() of the first piece in cat order (migration.py:538).
          rs_meta_slot ms;
          ms.name_id = name;
          ms.subfield = f;
          ms.src_rank = plan->ops[order[0]].src_rank;
          ms.first_is_self = ms.src_rank == rank ? 1 : 0;
          prog->meta.push_back(ms);
          continue;
        }
        rs_dst_slot ds;
        std::memset(&ds, 0, sizeof(ds));
        ds.name_id = name;
        ds.subfield = f;
        ds.ndim = full.ndim;
        for (int k = 0; k < full.ndim; ++k) ds.shape[k] = shape[k];
        ds.nbytes = (uint64_t)(numel * E);
        const int32_t dslot = (int32_t)prog->dst.size();
        prog->dst.push_back(ds);
        int64_t pos = 0;  // running offset along the slice dim inside the target
        for (size_t p = 0; p < order.size(); ++p) {
          const rs_op& op = plan->ops[order[p]];
          const Meta& sm = plan->src_meta_of_op[order[p]];
          const PieceGeom& g = geo[p];
          auto key = std::make_tuple(op.src_rank, name, f);
          auto it = src_slot_of.find(key);
          int32_t sslot;
          if (it == src_slot_of.end()) {
            rs_src_slot ss;
            std::memset(&ss, 0, sizeof(ss));
            ss.src_rank = op.src_rank;
            ss.name_id = name;
            ss.subfield = f;
            ss.nbytes = (uint64_t)(sm.numel() * E);
            sslot = (int32_t)prog->src.size();
            prog->src.push_back(ss);
            src_slot_of.emplace(key, sslot);
          } else {
            sslot = it->second;
          }
          rs_segment s;
          std::memset(&s, 0, sizeof(s));
          s.src_slot = sslot;
          s.dst_slot = dslot;
          if (!tp || (g.whole && order.size() == 1)) {
            s.src_offset = 0;
            s.dst_offset = 0;
            s.rows = 1;
            s.row_bytes = (uint64_t)(g.numel * E);
            s.src_pitch = s.row_bytes;
            s.dst_pitch = s.row_bytes;
          } else {
            const int64_t row = g.piece_extent * g.inner * E;
            s.rows = (uint64_t)g.outer;
            s.row_bytes = (uint64_t)row;
            s.src_pitch = (uint64_t)(g.src_extent * g.inner * E);
            s.dst_pitch = (uint64_t)(shape[d] * g.inner * E);
            s.src_offset = (uint64_t)(g.src_start * g.inner * E);
            s.dst_offset = (uint64_t)(pos * g.inner * E);
            if (s.rows == 1 || (s.src_pitch == s.row_bytes && s.dst_pitch == s.row_bytes)) {
              s.row_bytes *= s.rows;
              s.rows = 1;
              s.src_pitch = s.row_bytes;
              s.dst_pitch = s.row_bytes;
            }
          }
          pos += g.piece_extent;
          const uint64_t bytes = s.rows * s.row_bytes;
          if (op.src_rank == rank) prog->local_bytes += bytes; else prog->remote_bytes += bytes;
          if (bytes > 0) prog->segs.push_back(s);
        }
      }
    }
  } catch (const std::exception& e) {
    return fail_and_free(prog, RS_ERR_ARG, std::string("rs_program_build: ") + e.what());
  }
  *out = prog;
  return RS_OK;
}

int rs_program_counts_get(const rs_program* prog, rs_program_counts* out) {
  if (!prog || !out) return fail(RS_ERR_ARG, "rs_program_counts_get: NULL argument");
  out->n_dst_slots = (int64_t)prog->dst.size();
  out->n_src_slots = (int64_t)prog->src.size();
  out->n_meta_slots = (int64_t)prog->meta.size();
  out->n_segments = (int64_t)prog->segs.size();
  out->remote_bytes = prog->remote_bytes;
  out->local_bytes = prog->local_bytes;
  return RS_OK;
}

int rs_program_dst_slots(const rs_program* p, rs_dst_slot* o, int64_t c) {
  return p ? copy_out(p->dst, o, c, "rs_program_dst_slots") : fail(RS_ERR_ARG, "NULL program");
}
int rs_program_src_slots(const rs_program* p, rs_src_slot* o, int64_t c) {
  return p ? copy_out(p->src, o, c, "rs_program_src_slots") : fail(RS_ERR_ARG, "NULL program");
}
int rs_program_meta_slots(const rs_program* p, rs_meta_slot* o, int64_t c) {
  return p ? copy_out(p->meta, o, c, "rs_program_meta_slots") : fail(RS_ERR_ARG, "NULL program");
}
int rs_program_segments(const rs_program* p, rs_segment* o, int64_t c) {
  return p ? copy_out(p->segs, o, c, "rs_program_segments") : fail(RS_ERR_ARG, "NULL program");
}
void rs_program_free(rs_program* prog) { delete prog; }

}  // extern "C"

namespace {
int resolve_segments(const rs_program* prog, int32_t src_rank, const uint64_t* src_dev, const uint64_t* src_extent,
                     const uint64_t* dst_dev, const uint64_t* dst_extent, rs_copy_desc* out, int64_t capacity, int64_t* n_out) {
  int64_t k = 0;
  for (size_t i = 0; i < prog->segs.size(); ++i) {
    const rs_segment& s = prog->segs[i];
    if (src_rank >= 0 && prog->src[s.src_slot].src_rank != src_rank) continue;
    if (k >= capacity) return fail(RS_ERR_CAPACITY, "rs_program_resolve: capacity too small");
    // last byte touched = offset + (rows - 1) * pitch + row_bytes, computed without overflow.
    const unsigned __int128 send = (unsigned __int128)s.src_offset + (unsigned __int128)(s.rows - 1) * s.src_pitch + s.row_bytes;
    const unsigned __int128 dend = (unsigned __int128)s.dst_offset + (unsigned __int128)(s.rows - 1) * s.dst_pitch + s.row_bytes;
    if (s.row_bytes > s.src_pitch || s.row_bytes > s.dst_pitch || send > src_extent[s.src_slot] || dend > dst_extent[s.dst_slot])
      return fail(RS_ERR_BOUNDS, "rs_program_resolve: segment " + std::to_string(i) + " leaves its source or target (src slot " +
                                     std::to_string(s.src_slot) + " extent " + std::to_string(src_extent[s.src_slot]) + ", dst slot " +
                                     std::to_string(s.dst_slot) + " extent " + std::to_string(dst_extent[s.dst_slot]) + ")");
    if (!src_dev[s.src_slot] || !dst_dev[s.dst_slot])
      return fail(RS_ERR_ARG, "rs_program_resolve: NULL address for segment " + std::to_string(i));
    rs_copy_desc& c = out[k++];
    c.src_dev = src_dev[s.src_slot] + s.src_offset;
    c.dst_dev = dst_dev[s.dst_slot] + s.dst_offset;
    c.rows = s.rows;
    c.row_bytes = s.row_bytes;
    c.src_pitch = s.src_pitch;
    c.dst_pitch = s.dst_pitch;
    // remote: the copying rank (the source rank when filtered by it) is not the other end
    const int32_t copier = src_rank >= 0 ? src_rank : prog->rank;
    const int32_t other = src_rank >= 0 ? prog->rank : prog->src[s.src_slot].src_rank;
    c.flags = copier != other ? RS_COPY_REMOTE : 0u;
  }
  if (n_out) *n_out = k;
  return RS_OK;
}
}  // namespace

extern "C" {

int rs_program_resolve_from(const rs_program* prog, int32_t src_rank, const uint64_t* src_dev, const uint64_t* src_extent,
                            const uint64_t* dst_dev, const uint64_t* dst_extent, rs_copy_desc* out, int64_t capacity,
                            int64_t* n_out) {
  if (!prog || src_rank < 0) return fail(RS_ERR_ARG, "rs_program_resolve_from: bad argument");
  if (!prog->segs.empty() && (!src_dev || !src_extent || !dst_dev || !dst_extent || (!out && capacity > 0)))
    return fail(RS_ERR_ARG, "rs_program_resolve_from: NULL argument");
  return resolve_segments(prog, src_rank, src_dev, src_extent, dst_dev, dst_extent, out, capacity, n_out);
}

// Bind slots to addresses; every segment is bounds-checked against its slot extents.
int rs_program_resolve(const rs_program* prog, const uint64_t* src_dev, const uint64_t* src_extent,
                       const uint64_t* dst_dev, const uint64_t* dst_extent, rs_copy_desc* out, int64_t capacity) {
  if (!prog) return fail(RS_ERR_ARG, "rs_program_resolve: NULL program");
  if (capacity < (int64_t)prog->segs.size()) return fail(RS_ERR_CAPACITY, "rs_program_resolve: capacity too small");
  if (!prog->segs.empty() && (!src_dev || !src_extent || !dst_dev || !dst_extent || !out))
    return fail(RS_ERR_ARG, "rs_program_resolve: NULL argument");
  for (size_t i = 0; i < prog->segs.size(); ++i) {
    const rs_segment& s = prog->segs[i];
    // last byte touched = offset + (rows - 1) * pitch + row_bytes, computed without overflow.
    const unsigned __int128 send = (unsigned __int128)s.src_offset + (unsigned __int128)(s.rows - 1) * s.src_pitch + s.row_bytes;
    const unsigned __int128 dend = (unsigned __int128)s.dst_offset + (unsigned __int128)(s.rows - 1) * s.dst_pitch + s.row_bytes;
    if (s.row_bytes > s.src_pitch || s.row_bytes > s.dst_pitch || send > src_extent[s.src_slot] || dend > dst_extent[s.dst_slot])
      return fail(RS_ERR_BOUNDS, "rs_program_resolve: segment " + std::to_string(i) + " leaves its source or target (src slot " +
                                     std::to_string(s.src_slot) + " extent " + std::to_string(src_extent[s.src_slot]) + ", dst slot " +
                                     std::to_string(s.dst_slot) + " extent " + std::to_string(dst_extent[s.dst_slot]) + ")");
    if (!src_dev[s.src_slot] || !dst_dev[s.dst_slot])
      return fail(RS_ERR_ARG, "rs_program_resolve: NULL address for segment " + std::to_string(i));
    rs_copy_desc& c = out[i];
    c.src_dev = src_dev[s.src_slot] + s.src_offset;
    c.dst_dev = dst_dev[s.dst_slot] + s.dst_offset;
    c.rows = s.rows;
    c.row_bytes = s.row_bytes;
    c.src_pitch = s.src_pitch;
    c.dst_pitch = s.dst_pitch;
    c.flags = prog->src[s.src_slot].src_rank != prog->rank ? RS_COPY_REMOTE : 0u;
  }
  return RS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Interval planner (rs_plan_build_rules): layouts beyond the reference's contiguous chunks.
// ---------------------------------------------------------------------------------------------
namespace {

struct Span {
  int64_t lo, hi;   // full-tensor coordinates along the slice dim
  int64_t at;       // storage position of lo inside the shard
};

// Slice-dim intervals held by a shard, in storage order.
int shard_spans(const Meta& m, int d, const Rule* rule, std::vector<Span>& out) {
  out.clear();
  const int64_t F = m.shape[d];
  if (!m.is_tp()) {
    out.push_back({0, F, 0});
    return RS_OK;
  }
  const int64_t i = m.tp_index, T = m.tp_deg;
  if (!rule || rule->n_groups == 0) {
    if (F % T) return fail(RS_ERR_SHAPE, "slice dim extent not divisible by tp degree: " + meta_str(m));
    out.push_back({i * F / T, (i + 1) * F / T, 0});
    return RS_OK;
  }
  int64_t at = 0;
  for (int g = 0; g < rule->n_groups; ++g) {
    const rs_slice_group& G = rule->groups[g];
    if (G.units <= 0 || G.size <= 0 || G.size % G.units || G.offset < 0 || G.offset + G.size > F)
      return fail(RS_ERR_SHAPE, "malformed slice rule group for " + meta_str(m));
    const int64_t usz = G.size / G.units;
    int64_t u0, nu;
    if (G.units >= T) {
      if (G.units % T) return fail(RS_ERR_SHAPE, "group units not divisible by tp degree: " + meta_str(m));
      nu = G.units / T;
      u0 = i * nu;
    } else {
      if (T % G.units) return fail(RS_ERR_SHAPE, "tp degree not a multiple of group units: " + meta_str(m));
      nu = 1;
      u0 = i * G.units / T;
    }
    out.push_back({G.offset + u0 * usz, G.offset + (u0 + nu) * usz, at});
    at += nu * usz;
  }
  return RS_OK;
}

int64_t spans_extent(const std::vector<Span>& v) {
  int64_t e = 0;
  for (const Span& s : v) e += s.hi - s.lo;
  return e;
}

}  // namespace

extern "C" {

int rs_plan_build_rules(const rs_rank_layout* src, int32_t n_src, const rs_rank_layout* dst, int32_t n_dst,
                        const rs_slice_rule* rules, int32_t n_rules, const rs_plan_opts* opts, rs_plan** out) {
  if (!out) return fail(RS_ERR_ARG, "rs_plan_build_rules: out is NULL");
  *out = nullptr;
  if (n_rules < 0 || (n_rules > 0 && !rules)) return fail(RS_ERR_ARG, "rs_plan_build_rules: bad rule array");
  rs_plan* plan = new (std::nothrow) rs_plan();
  if (!plan) return fail(RS_ERR_ARG, "rs_plan_build_rules: out of host memory");
  plan->mode = 1;
  plan->order = RS_ORDER_SEMANTIC;
  try {
    int rc = load_layout(src, n_src, plan->src, "source layout");
    if (rc) { delete plan; return rc; }
    rc = load_layout(dst, n_dst, plan->dst, "target layout");
    if (rc) { delete plan; return rc; }
    std::unordered_map<int32_t, Rule> rule_of;
    for (int32_t r = 0; r < n_rules; ++r) {
      if (rules[r].n_groups < 0 || rules[r].n_groups > RS_MAX_GROUPS)
        return fail_and_free(plan, RS_ERR_ARG, "rs_plan_build_rules: a rule has more than RS_MAX_GROUPS groups");
      Rule R;
      R.n_groups = rules[r].n_groups;
      for (int g = 0; g < R.n_groups; ++g) R.groups[g] = rules[r].groups[g];
      rule_of[rules[r].name_id] = R;
    }
    (void)opts;  // the interval planner always writes slice order and balances replicas
    int32_t max_rank = 0;
    for (const RankLayout& L : plan->src) max_rank = std::max(max_rank, L.rank);
    std::vector<double> egress((size_t)max_rank + 1, 0.0);
    std::vector<Span> dspans, sspans;
    struct Owner { int32_t rank; const Meta* meta; std::vector<Span> spans; };
    std::vector<Owner> owners;
    for (const RankLayout& D : plan->dst) {
      for (const Meta& dm : D.tensors) {
        auto rit = rule_of.find(dm.name);
        const Rule* rule = rit == rule_of.end() ? nullptr : &rit->second;
        owners.clear();
        for (const RankLayout& S : plan->src) {
          auto it = S.by_name.find(dm.name);
          if (it != S.by_name.end()) owners.push_back({S.rank, &S.tensors[it->second], {}});
        }
        if (owners.empty())
          return fail_and_free(plan, RS_ERR_NO_OWNER, "target param " + meta_str(dm) + " of rank " + std::to_string(D.rank) +
                                                         " is not present in any source");
        // The working dim: the target's slice dim, else any source's; all TP metas must agree.
        int d = -1;
        int32_t raw_dim = RS_NO_SLICE;
        auto take_dim = [&](const Meta& m) -> bool {
          if (!m.is_tp()) return true;
          if (raw_dim == RS_NO_SLICE) { raw_dim = m.slice_dim; d = m.norm_dim(); return true; }
          return m.norm_dim() == d;
        };
        if (!take_dim(dm)) return fail_and_free(plan, RS_ERR_SLICE_DIM, "slice dim mismatch for " + meta_str(dm));
        for (const Owner& o : owners)
          if (!take_dim(*o.meta) || o.meta->ndim != dm.ndim)
            return fail_and_free(plan, RS_ERR_SLICE_DIM, "slice dim mismatch between " + meta_str(*o.meta) + " and " + meta_str(dm));
        for (const Owner& o : owners)
          for (int k = 0; k < dm.ndim; ++k)
            if (o.meta->shape[k] != dm.shape[k])
              return fail_and_free(plan, RS_ERR_SHAPE, "full shape mismatch between " + meta_str(*o.meta) + " and " + meta_str(dm));
        Piece base;
        base.name = dm.name;
        base.dst_rank = D.rank;
        base.ndim = dm.ndim;
        for (int k = 0; k < dm.ndim; ++k) base.dst_shape[k] = dm.shape[k];
        if (d < 0) {  // replicated everywhere: whole-tensor copies
          base.inner = dm.full_numel();
          base.src_numel = base.inner;
          int32_t best = -1;
          for (const Owner& o : owners)
            if (o.rank == D.rank) best = o.rank;
          if (best < 0)
            for (const Owner& o : owners)
              if (best < 0 || egress[o.rank] < egress[best]) best = o.rank;
          base.src_rank = best;
          egress[best] += (double)base.inner * dm.itemsize;
          plan->pieces.push_back(base);
          continue;
        }
        for (int k = 0; k < d; ++k) base.outer *= dm.shape[k];
        for (int k = d + 1; k < dm.ndim; ++k) base.inner *= dm.shape[k];
        rc = shard_spans(dm, d, rule, dspans);
        if (rc) { delete plan; return rc; }
        base.dst_extent = spans_extent(dspans);
        base.dst_shape[d] = base.dst_extent;
        for (Owner& o : owners) {
          rc = shard_spans(*o.meta, d, rule, o.spans);
          if (rc) { delete plan; return rc; }
        }
        for (const Span& ds : dspans) {
          int64_t a = ds.lo;
          while (a < ds.hi) {
            // Owners holding index a, and how far each holds it contiguously (within this span).
            int64_t b = ds.hi;
            for (const Owner& o : owners)
              for (const Span& sp : o.spans) {
                if (sp.lo > a && sp.lo < b) b = sp.lo;  // another owner's span starts inside: cut there
                if (sp.lo <= a && a < sp.hi && sp.hi < b) b = sp.hi;
              }
            int32_t best = -1;
            const Owner* bo = nullptr;
            const Span* bs = nullptr;
            for (const Owner& o : owners)
              for (const Span& sp : o.spans)
                if (sp.lo <= a && b <= sp.hi) {
                  const bool self = o.rank == D.rank;
                  if (best < 0 || (self && best != D.rank) ||
                      (best != D.rank && !self && egress[o.rank] < egress[best])) {
                    best = o.rank; bo = &o; bs = &sp;
                  }
                }
            if (best < 0)
              return fail_and_free(plan, RS_ERR_NO_OWNER, "no source holds slice [" + std::to_string(a) + ", " + std::to_string(b) +
                                                             ") of " + meta_str(dm) + " for rank " + std::to_string(D.rank));
            Piece pc = base;
            pc.src_rank = best;
            pc.src_extent = spans_extent(bo->spans);
            pc.src_numel = pc.outer * pc.src_extent * pc.inner;
            pc.src_start = bs->at + (a - bs->lo);
            pc.dst_start = ds.at + (a - ds.lo);
            pc.len = b - a;
            egress[best] += (double)(pc.outer * pc.len * pc.inner * dm.itemsize);
            Piece* prev = plan->pieces.empty() ? nullptr : &plan->pieces.back();
            if (prev && prev->dst_rank == pc.dst_rank && prev->name == pc.name && prev->src_rank == pc.src_rank &&
                prev->src_start + prev->len == pc.src_start && prev->dst_start + prev->len == pc.dst_start) {
              prev->len += pc.len;  // contiguous in both shards: one piece
            } else {
              plan->pieces.push_back(pc);
            }
            a = b;
          }
        }
      }
    }
    // One rs_op per piece, for inspection (numel = elements of the piece).
    for (const Piece& pc : plan->pieces) {
      rs_op op;
      std::memset(&op, 0, sizeof(op));
      op.name_id = pc.name;
      op.src_rank = pc.src_rank;
      op.dst_rank = pc.dst_rank;
      op.src_slice_dim = op.dst_slice_dim = RS_NO_SLICE;
      op.src_tp_deg = op.dst_tp_deg = 1;
      op.numel = pc.outer * pc.len * pc.inner;
      plan->ops.push_back(op);
    }
  } catch (const std::exception& e) {
    return fail_and_free(plan, RS_ERR_ARG, std::string("rs_plan_build_rules: ") + e.what());
  }
  *out = plan;
  return RS_OK;
}

}  // extern "C"
