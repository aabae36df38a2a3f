// Activation exchange between adjacent pipeline stages whose DP/TP shapes differ.
//
// Restates what PipelineExecModule._get_recv_or_send_P2P_ops (Suika/pipeline_parallel.py:665-776)
// and the receive side's TP all-gather (Suika/pipeline_parallel.py:780-836) deliver, as the set of
// byte pieces each receiver ends up holding, so that one copy launch can write them straight into
// place:
//   - a receiver in DP group g of the next stage needs the batch rows [l_g, r_g) of the global
//     micro-batch; every DP group h of the sending stage that holds rows overlapping them supplies
//     the overlap (pipeline_parallel.py:711-721);
//   - along the slice dim the overlap is cut into k = max(s, d) equal chunks, s and d being the TP
//     degrees of groups h and g; chunk c comes from TP rank c * s / k of group h. In the reference
//     receiver j fetches its own share of the chunks by P2P (pipeline_parallel.py:723-742) and the
//     TP all-gather hands every receiver of group g the shares of the others (:817-832); the
//     union is all k chunks, each from that sender;
//   - rows that no sender covers are not written (the reference leaves them as the caller made
//     them).
// The sending stage's TP ranks hold the same activation, so which one supplies a chunk decides
// the load, not the bytes; the choice above is the reference's so that results stay identical
// even if they did not.

#include "../../include/suika_reshard.h"
#include "internal.h"

#include <algorithm>
#include <cstdint>
#include <exception>
#include <string>
#include <vector>

using suika_rs::fail;

namespace {

struct Mesh {
  std::vector<std::vector<int32_t>> groups;
  std::vector<int64_t> bsz;
  std::vector<int64_t> start;  // global first batch row of each group
};

int read_mesh(const rs_stage_mesh* m, const char* what, Mesh& out) {
  if (!m || m->n_groups < 0 || (m->n_groups > 0 && (!m->group_start || !m->ranks || !m->local_bsz)))
    return fail(RS_ERR_ARG, std::string(what) + ": malformed stage mesh");
  out.groups.resize(m->n_groups);
  out.bsz.resize(m->n_groups);
  out.start.resize(m->n_groups);
  int64_t row = 0;
  for (int g = 0; g < m->n_groups; ++g) {
    int32_t a = m->group_start[g], b = m->group_start[g + 1];
    if (a < 0 || b <= a) return fail(RS_ERR_ARG, std::string(what) + ": empty or unordered TP group " + std::to_string(g));
    out.groups[g].assign(m->ranks + a, m->ranks + b);
    for (int32_t r : out.groups[g])
      if (r < 0) return fail(RS_ERR_ARG, std::string(what) + ": negative rank");
    if (m->local_bsz[g] < 0) return fail(RS_ERR_ARG, std::string(what) + ": negative local batch size");
    out.bsz[g] = m->local_bsz[g];
    out.start[g] = row;  // pipeline_parallel.py:708-709: prefix sums of the local batch sizes
    row += m->local_bsz[g];
  }
  return RS_OK;
}

bool pow2(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }

// DP group of a rank within a stage; -1 when the rank is not in it.
int rank_group(const Mesh& m, int32_t rank) {
  for (size_t g = 0; g < m.groups.size(); ++g)
    for (int32_t r : m.groups[g])
      if (r == rank) return static_cast<int>(g);
  return -1;
}

int plan(const Mesh& src, const Mesh& dst, int64_t slice_size, std::vector<rs_act_piece>& out) {
  if (slice_size <= 0) return fail(RS_ERR_ARG, "slice dim has no elements");
  for (size_t dg = 0; dg < dst.groups.size(); ++dg) {
    const int64_t d = static_cast<int64_t>(dst.groups[dg].size());
    for (int64_t j = 0; j < d; ++j) {
      const int32_t receiver = dst.groups[dg][j];
      for (size_t sg = 0; sg < src.groups.size(); ++sg) {
        const int64_t lo = std::max(src.start[sg], dst.start[dg]);
        const int64_t hi = std::min(src.start[sg] + src.bsz[sg], dst.start[dg] + dst.bsz[dg]);
        if (lo >= hi) continue;  // pipeline_parallel.py:719-720
        const int64_t s = static_cast<int64_t>(src.groups[sg].size());
        // The reference's chunk arithmetic (:724-742, :824) tiles the slice dim only when one
        // degree divides the other (DeviceMesh2D.validate requires powers of two) and the
        // slice dim divides into the finer degree; otherwise parts would be left unwritten.
        if (!pow2(s) || !pow2(d))
          return fail(RS_ERR_SHAPE, "TP degrees " + std::to_string(s) + " and " + std::to_string(d) +
                                        " must be powers of two (device_mesh.py:192)");
        const int64_t k = std::max(s, d);
        if (slice_size % k != 0)
          return fail(RS_ERR_SHAPE, "slice dim of " + std::to_string(slice_size) + " does not divide into " +
                                        std::to_string(k) + " TP chunks");
        const int64_t chunk = slice_size / k;
        for (int64_t c = 0; c < k; ++c) {
          rs_act_piece p{};
          p.src_rank = src.groups[sg][c * s / k];
          p.dst_rank = receiver;
          p.src_batch = lo - src.start[sg];
          p.dst_batch = lo - dst.start[dg];
          p.n_batch = hi - lo;
          p.slice_start = c * chunk;
          p.slice_len = chunk;
          out.push_back(p);
        }
      }
    }
  }
  return RS_OK;
}

}  // namespace

extern "C" {

int rs_act_plan(const rs_stage_mesh* src, const rs_stage_mesh* dst, int64_t slice_size,
                rs_act_piece* out, int64_t capacity, int64_t* n_out) {
  try {
    if (!n_out) return fail(RS_ERR_ARG, "n_out is NULL");
    Mesh ms, md;
    int rc = read_mesh(src, "source stage", ms);
    if (rc != RS_OK) return rc;
    rc = read_mesh(dst, "target stage", md);
    if (rc != RS_OK) return rc;
    std::vector<rs_act_piece> pieces;
    rc = plan(ms, md, slice_size, pieces);
    if (rc != RS_OK) return rc;
    *n_out = static_cast<int64_t>(pieces.size());
    if (!out) return RS_OK;
    if (capacity < *n_out) return fail(RS_ERR_CAPACITY, "piece buffer holds " + std::to_string(capacity) +
                                                            " of " + std::to_string(*n_out));
    for (size_t i = 0; i < pieces.size(); ++i) out[i] = pieces[i];
    return RS_OK;
  } catch (const std::exception& e) {
    return fail(RS_ERR_ARG, std::string("rs_act_plan: ") + e.what());
  }
}

int rs_act_resolve(const rs_stage_mesh* src, const rs_stage_mesh* dst, const rs_act_geometry* geo,
                   const rs_act_piece* pieces, int64_t n_pieces,
                   const uint64_t* src_dev, const uint64_t* dst_dev, int32_t n_ranks,
                   rs_copy_desc* out, int64_t capacity, int64_t* n_out) {
  try {
    if (!geo || !n_out || (n_pieces > 0 && (!pieces || !src_dev || !dst_dev)) || n_pieces < 0 || n_ranks < 0)
      return fail(RS_ERR_ARG, "rs_act_resolve: NULL or negative argument");
    Mesh ms, md;
    int rc = read_mesh(src, "source stage", ms);
    if (rc != RS_OK) return rc;
    rc = read_mesh(dst, "target stage", md);
    if (rc != RS_OK) return rc;
    const int nd = geo->ndim, bd = geo->batch_dim, sd = geo->slice_dim;
    if (nd < 2 || nd > RS_MAX_DIMS || bd < 0 || bd >= nd || sd < 0 || sd >= nd || bd == sd || geo->elem_bytes <= 0)
      return fail(RS_ERR_ARG, "activation geometry: need 2..8 dims and distinct batch and slice dims");
    for (int i = 0; i < nd; ++i)
      if (i != bd && geo->shape[i] < 0) return fail(RS_ERR_ARG, "activation geometry: negative extent");
    // Element (o, a, m, b, i) with a the outer and b the inner of the two cut dims:
    //   outer = prod(shape[:min]), mid = prod(shape[min+1:max]), inner = prod(shape[max+1:]).
    const int lo_dim = std::min(bd, sd), hi_dim = std::max(bd, sd);
    int64_t outer = 1, mid = 1, inner = 1;
    for (int i = 0; i < lo_dim; ++i) outer *= geo->shape[i];
    for (int i = lo_dim + 1; i < hi_dim; ++i) mid *= geo->shape[i];
    for (int i = hi_dim + 1; i < nd; ++i) inner *= geo->shape[i];
    const int64_t S = geo->shape[sd];
    const uint64_t e = static_cast<uint64_t>(geo->elem_bytes);
    const bool batch_outer = bd < sd;

    int64_t n = 0;
    for (int64_t p = 0; p < n_pieces; ++p) {
      const rs_act_piece& pc = pieces[p];
      if (pc.src_rank < 0 || pc.src_rank >= n_ranks || pc.dst_rank < 0 || pc.dst_rank >= n_ranks)
        return fail(RS_ERR_ARG, "piece " + std::to_string(p) + " names a rank outside the address tables");
      const uint64_t sbase = src_dev[pc.src_rank], dbase = dst_dev[pc.dst_rank];
      if (!sbase || !dbase)
        return fail(RS_ERR_ARG, "piece " + std::to_string(p) + ": no address for rank " +
                                    std::to_string(sbase ? pc.dst_rank : pc.src_rank));
      const int sg = rank_group(ms, pc.src_rank), dg = rank_group(md, pc.dst_rank);
      if (sg < 0 || dg < 0) return fail(RS_ERR_ARG, "piece " + std::to_string(p) + ": rank not in its stage");
      const int64_t Bs = ms.bsz[sg], Bd = md.bsz[dg];
      if (pc.n_batch < 0 || pc.src_batch < 0 || pc.dst_batch < 0 || pc.src_batch + pc.n_batch > Bs ||
          pc.dst_batch + pc.n_batch > Bd || pc.slice_start < 0 || pc.slice_len < 0 || pc.slice_start + pc.slice_len > S)
        return fail(RS_ERR_BOUNDS, "piece " + std::to_string(p) + " leaves its tensors");
      if (pc.n_batch == 0 || pc.slice_len == 0 || mid == 0 || inner == 0) continue;
      for (int64_t o = 0; o < outer; ++o) {
        rs_copy_desc d{};
        if (batch_outer) {
          // rows run over (batch, mid); one row = the slice chunk x inner
          d.rows = static_cast<uint64_t>(pc.n_batch * mid);
          d.row_bytes = static_cast<uint64_t>(pc.slice_len * inner) * e;
          d.src_pitch = d.dst_pitch = static_cast<uint64_t>(S * inner) * e;
          d.src_dev = sbase + static_cast<uint64_t>(((o * Bs + pc.src_batch) * mid * S + pc.slice_start) * inner) * e;
          d.dst_dev = dbase + static_cast<uint64_t>(((o * Bd + pc.dst_batch) * mid * S + pc.slice_start) * inner) * e;
        } else {
          // rows run over (slice, mid); one row = the batch range x inner
          d.rows = static_cast<uint64_t>(pc.slice_len * mid);
          d.row_bytes = static_cast<uint64_t>(pc.n_batch * inner) * e;
          d.src_pitch = static_cast<uint64_t>(Bs * inner) * e;
          d.dst_pitch = static_cast<uint64_t>(Bd * inner) * e;
          d.src_dev = sbase + static_cast<uint64_t>(((o * S + pc.slice_start) * mid * Bs + pc.src_batch) * inner) * e;
          d.dst_dev = dbase + static_cast<uint64_t>(((o * S + pc.slice_start) * mid * Bd + pc.dst_batch) * inner) * e;
        }
        d.flags = pc.src_rank != pc.dst_rank ? RS_COPY_REMOTE : 0u;
        if (out) {
          if (n >= capacity) return fail(RS_ERR_CAPACITY, "descriptor buffer too small");
          out[n] = d;
        }
        ++n;
      }
    }
    *n_out = n;
    return RS_OK;
  } catch (const std::exception& e) {
    return fail(RS_ERR_ARG, std::string("rs_act_resolve: ") + e.what());
  }
}

}  // extern "C"
