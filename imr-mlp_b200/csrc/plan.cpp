// plan.cpp -- host-side model planning: graph validation, basis-shape
// selection, kernel slot map, moment-graph program and cell preparation.
#include "plan.hpp"

#include <algorithm>
#include <cmath>
#include <numeric>
#include <unordered_set>

namespace mtpb {

// Moment-graph checks of MLIPCore::setup_from_text
// (runtime/mtp/mlip.cpp:700-760): every rule input defined before use, no
// cycles, no accumulation into a target after it was consumed, scalars map to
// defined moments.
bool validate_model(const ModelHost &m, std::string *err)
{
    auto fail = [&](const std::string &s) {
        if (err)
            *err = "invalid MTP model: " + s;
        return false;
    };
    if (m.K <= 0 || m.K > 64)
        return fail("species_count must be in 1..64");
    if (m.mu <= 0 || m.R <= 0 || m.R > 64)
        return fail("radial_funcs_count and radial_basis_size must be positive (R <= 64)");
    const int pairs = m.split ? m.K * m.K : 1;
    if ((int)m.min_dist.size() != pairs || (int)m.max_dist.size() != pairs)
        return fail("radial interval count does not match the split flag");
    for (int p = 0; p < pairs; ++p)
        if (!(m.max_dist[p] > m.min_dist[p]) || !std::isfinite(m.max_dist[p]) ||
            !std::isfinite(m.min_dist[p]) || m.min_dist[p] < 0)
            return fail("invalid radial interval");
    if (!std::isfinite(m.scaling))
        return fail("scaling must be finite");
    // radial families: the checks of the reference's loaders and constructors
    // (runtime/mtp/radial_basis.h:46-200, basis/cutoff.cpp, basis/xtrans.cpp)
    if (!m.family.empty() && (int)m.family.size() != pairs)
        return fail("radial family count does not match the split flag");
    for (int p = 0; p < (int)m.family.size(); ++p) {
        const RadialFamily &f = m.family[p];
        const double lo = m.min_dist[p], hi = m.max_dist[p];
        if (f.type < RB_CHEBYSHEV || f.type > RB_POLYB_COS)
            return fail("unsupported radial basis type " + std::to_string(f.type) +
                        " (RBChebyshev, RBChebyCos, RBChebyshevPoly4/5, "
                        "RBChebyshevConfigurable, RBPolyB and RBPolyBCos are implemented)");
        if (f.type == RB_POLYB || f.type == RB_POLYB_COS) {
            if (f.poly_matrix.size() != (size_t)m.R * m.R || f.poly_norm.size() != (size_t)m.R)
                return fail("RBPolyB needs an R x R matrix and R normalisations");
            for (double v : f.poly_matrix)
                if (!std::isfinite(v))
                    return fail("non-finite RBPolyB orthogonalisation matrix");
            for (double v : f.poly_norm)
                if (!std::isfinite(v) || !(v > 0))
                    return fail("invalid RBPolyB normalisation");
        }
        if (!std::isfinite(f.b) || !std::isfinite(f.r1) || !std::isfinite(f.r2) ||
            !std::isfinite(f.lambda) || !std::isfinite(f.scale_lambda))
            return fail("non-finite radial parameter");
        if (f.type != RB_CONFIGURABLE)
            continue;
        if (f.cutoff < CUT_QUADRATIC || f.cutoff > CUT_SMOOTHSTEP7 || f.shift < SHIFT_LINEAR ||
            f.shift > SHIFT_EXPONENTIAL_TANH)
            return fail("unknown configurable cutoff_type or shift_type");
        if (f.cutoff == CUT_SMOOTHSTEP7 && !(lo < f.r1 && f.r1 <= f.r2 && f.r2 < hi))
            return fail("smoothstep7 cutoff requires min_dist < cutoff_r1 <= cutoff_r2 < max_dist");
        if ((f.shift == SHIFT_EXPONENTIAL || f.shift == SHIFT_EXPONENTIAL_LEFT ||
             f.shift == SHIFT_EXPONENTIAL_TANH) &&
            f.lambda != 0.0 && !(std::isfinite(std::expm1(f.lambda)) && std::expm1(f.lambda) != 0.0))
            return fail("shift_lambda produces a non-finite exponential normalization");
        if (f.shift == SHIFT_EXPONENTIAL_TANH && f.scale_lambda != 0.0 &&
            std::tanh(f.scale_lambda) == 0.0)
            return fail("shift_scale_lambda produces an invalid normalization");
    }
    const int nb = m.nb(), M = m.M;
    if (nb <= 0 || nb > M)
        return fail("basic moment count exceeds total moment slots");
    for (int i = 0; i < nb; ++i) {
        const int *b = &m.basic[4 * i];
        if (b[0] < 0 || b[0] >= m.mu || b[1] < 0 || b[2] < 0 || b[3] < 0)
            return fail("invalid basic moment index");
    }
    std::vector<char> defined(M, 0), consumed(M, 0);
    for (int i = 0; i < nb; ++i)
        defined[i] = 1;
    for (int t = 0; t < m.T(); ++t) {
        const int *r = &m.times[4 * t];
        const int l1 = r[0], l2 = r[1], id = r[3];
        if (l1 < 0 || l1 >= M || l2 < 0 || l2 >= M || id < nb || id >= M || !defined[l1] ||
            !defined[l2] || id == l1 || id == l2 || consumed[id])
            return fail("moment graph has an undefined input, cycle or late accumulation");
        defined[id] = 1;
        consumed[l1] = 1;
        consumed[l2] = 1;
    }
    for (int s = 0; s < m.S(); ++s) {
        const int x = m.mapping[s];
        if (x < 0 || x >= M || !defined[x])
            return fail("scalar maps to an undefined moment");
    }
    if ((int)m.radial.size() != m.K * m.K * m.mu * m.R || (int)m.species.size() != m.K ||
        (int)m.moment.size() != m.S())
        return fail("coefficient array sizes do not match the model");
    for (double v : m.radial)
        if (!std::isfinite(v))
            return fail("radial coefficients must be finite");
    for (double v : m.species)
        if (!std::isfinite(v))
            return fail("species coefficients must be finite");
    for (double v : m.moment)
        if (!std::isfinite(v))
            return fail("moment coefficients must be finite");
    return true;
}

// Smallest instantiated shape whose complete tensors contain every basic
// moment of the model.
int select_shape(const ModelHost &m, std::string *err)
{
    std::vector<int> need(m.mu, -1);
    for (int i = 0; i < m.nb(); ++i) {
        const int *b = &m.basic[4 * i];
        need[b[0]] = std::max(need[b[0]], b[1] + b[2] + b[3]);
    }
    int best = -1, best_slots = 1 << 30;
    for (int id = 0; id < SHAPE_COUNT; ++id) {
        const ShapeDesc &d = shape_desc(id);
        bool ok = true;
        for (int mu = 0; mu < m.mu && ok; ++mu)
            if (need[mu] >= 0 && (mu >= d.nmu || d.numax[mu] < need[mu]))
                ok = false;
        if (ok && d.nslot < best_slots) {
            best = id;
            best_slots = d.nslot;
        }
    }
    if (best < 0 && err) {
        std::string s = "basis shape not supported by the compiled kernels; max degree per "
                        "radial channel:";
        for (int v : need)
            s += " " + std::to_string(v);
        *err = s;
    }
    return best;
}

bool build_slot_map(const ModelHost &m, int shape, std::vector<int> &slot_of_basic,
                    std::string *err)
{
    slot_of_basic.assign(m.nb(), -1);
    std::vector<char> used(shape_desc(shape).nslot, 0);
    for (int i = 0; i < m.nb(); ++i) {
        const int *b = &m.basic[4 * i];
        const int s = shape_slot(shape, b[0], b[1], b[2], b[3]);
        if (s < 0) {
            if (err)
                *err = "basic moment outside the selected kernel shape";
            return false;
        }
        if (used[s]) {
            if (err)
                *err = "duplicate basic moment in alpha_index_basic";
            return false;
        }
        used[s] = 1;
        slot_of_basic[i] = s;
    }
    return true;
}

namespace {

struct Item {
    std::vector<DagRec> recs;
    int energy = -1;   // energy_moments index of the item's ENERGY record
};

// Longest-processing-time assignment of items to the plan's streams, then
// padding to equal length.  Appends the phase to plan.recs.
void emit_packed(const std::vector<Item> &items, DagPlan &plan)
{
    std::vector<int> order(items.size());
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
        return items[a].recs.size() > items[b].recs.size();
    });
    const int S = plan.streams;
    std::vector<std::vector<DagRec>> streams(S);
    std::vector<std::vector<int>> energy(S);
    std::vector<size_t> load(S, 0);
    for (int idx : order) {
        int s = (int)(std::min_element(load.begin(), load.end()) - load.begin());
        for (const DagRec &r : items[idx].recs) {
            streams[s].push_back(r);
            energy[s].push_back(((r.outf >> 16) & DAG_ENERGY) ? items[idx].energy : -1);
        }
        load[s] += items[idx].recs.size();
    }
    size_t len = *std::max_element(load.begin(), load.end());
    const DagRec pad = make_rec(plan.zero_row, plan.zero_row, 0, 0, 0.0);
    for (size_t r = 0; r < len; ++r)
        for (int s = 0; s < S; ++s) {
            const bool real = r < streams[s].size();
            plan.recs.push_back(real ? streams[s][r] : pad);
            plan.rec_energy.push_back(real ? energy[s][r] : -1);
        }
    plan.phase_rows.push_back((int)len);
}

// Emits one phase of independent items.  An item much longer than the even
// share ceil(records / streams) would set the phase length alone, so it is
// split into parts of about that share, each summed into a partial row, and a
// following combine phase adds the partial rows (times the constant one row,
// as operand two so that the dual graph keeps it (1, 0)) and ends with the
// item's original flags.  Partial rows come from `pool` and are reused by later
// phases.  Returns the number of phases emitted (1 or 2).
int emit_phase(std::vector<Item> &items, DagPlan &plan, std::vector<int> &pool)
{
    size_t total = 0, longest = 0;
    for (const Item &it : items) {
        total += it.recs.size();
        longest = std::max(longest, it.recs.size());
    }
    const size_t S = (size_t)plan.streams;
    const size_t share = std::max<size_t>(4, (total + S - 1) / S);
    // splitting saves about len - share rows of this phase and costs the
    // combine phase (one row per part) plus a barrier
    auto split = [&](size_t len) { return len > share + (len + share - 1) / share + 1; };
    if (!split(longest)) {
        emit_packed(items, plan);
        return 1;
    }
    std::vector<Item> parts, combine;
    size_t used = 0;
    for (Item &it : items) {
        if (!split(it.recs.size())) {
            parts.push_back(std::move(it));
            continue;
        }
        // the item's closing record keeps its flags in the combine item; a
        // pure flag record (zero x zero, e.g. the energy term) moves there
        DagRec last = it.recs.back();
        std::vector<DagRec> body(it.recs.begin(), it.recs.end() - 1);
        const bool flag_only = last.s12 == ((unsigned)plan.zero_row | ((unsigned)plan.zero_row << 16));
        if (!flag_only) {
            DagRec plain = last;
            plain.outf = 0;
            body.push_back(plain);
        }
        const size_t k = (body.size() + share - 1) / share;
        const size_t per = (body.size() + k - 1) / k;
        Item comb;
        comb.energy = it.energy;
        for (size_t j = 0; j * per < body.size(); ++j) {
            if (used == pool.size())
                pool.push_back(plan.nrows++);
            const int prow = pool[used++];
            Item part;
            const size_t e = std::min(body.size(), (j + 1) * per);
            part.recs.assign(body.begin() + j * per, body.begin() + e);
            part.recs.back().outf = (unsigned)prow | ((unsigned)DAG_END << 16);
            parts.push_back(std::move(part));
            comb.recs.push_back(make_rec(prow, plan.one_row, 0, 0, 1.0));
        }
        if (flag_only)
            comb.recs.push_back(last);
        else
            comb.recs.back().outf = last.outf;
        combine.push_back(std::move(comb));
    }
    emit_packed(parts, plan);
    emit_packed(combine, plan);
    return 2;
}

} // namespace

// Builds the record program executed by k_dag (efs.cu).  Forward phases follow
// the forward product rules level by level (potential_mtp.cpp:2914-2921 order
// within a target), accumulating the linear energy of scalar moments
// (:2966-2970).  Reverse phases compute the adjoint of every moment that is a
// rule operand, by decreasing level, as a sum over its uses (the gather form
// of backpropagate_moments, :3292-3305), and finally the adjoints of the basic
// moments, written to the kernel slots.
static bool build_dag_plan_streams(const ModelHost &m, int shape,
                                   const std::vector<int> &slot_of_basic, int streams,
                                   DagPlan &plan, std::string *err)
{
    const int nb = m.nb(), M = m.M, T = m.T();
    const int nslot = shape_desc(shape).nslot;
    std::vector<int> level(M, 0);
    std::vector<char> is_operand(M, 0), is_target(M, 0);
    for (int t = 0; t < T; ++t) {
        const int *r = &m.times[4 * t];
        level[r[3]] = std::max(level[r[3]], std::max(level[r[0]], level[r[1]]) + 1);
        is_operand[r[0]] = is_operand[r[1]] = 1;
        is_target[r[3]] = 1;
    }
    int maxlevel = 0;
    for (int x = 0; x < M; ++x)
        maxlevel = std::max(maxlevel, level[x]);
    std::vector<double> scal(M, 0.0);
    std::vector<char> is_scalar(M, 0);
    for (int s = 0; s < m.S(); ++s) {
        scal[m.mapping[s]] += m.moment[s];
        is_scalar[m.mapping[s]] = 1;
    }
    std::vector<int> energy_index(M, -1), energy_moments;
    for (int x = 0; x < M; ++x)
        if (is_scalar[x]) {
            energy_index[x] = (int)energy_moments.size();
            energy_moments.push_back(x);
        }
    // rows: kernel slots, operand targets, their adjoints, constants
    std::vector<int> row(M, -1), adjrow(M, -1);
    for (int i = 0; i < nb; ++i)
        row[i] = slot_of_basic[i];
    int next = nslot;
    for (int x = nb; x < M; ++x)
        if (is_target[x] && is_operand[x])
            row[x] = next++;
    for (int x = nb; x < M; ++x)
        if (row[x] >= 0)
            adjrow[x] = next++;
    plan = DagPlan{};
    plan.one_row = next++;
    plan.zero_row = next++;
    plan.scratch_row = next++;
    plan.nrows = next;
    plan.energy_moments = energy_moments;
    plan.streams = streams;
    if (plan.nrows >= 65535) {   // the dual graph adds one row
        if (err)
            *err = "moment graph too large for 16-bit row indices (" +
                   std::to_string(plan.nrows) + " rows)";
        return false;
    }
    // rules grouped by target, in file order
    std::vector<std::vector<int>> rules_of(M);
    for (int t = 0; t < T; ++t)
        rules_of[m.times[4 * t + 3]].push_back(t);

    // ---- forward phases ----------------------------------------------------
    const int nfwd = std::max(1, maxlevel);
    std::vector<int> pool;   // partial rows of split items
    int nfwd_phases = 0;
    for (int L = 1; L <= nfwd; ++L) {
        std::vector<Item> items;
        if (L == 1) {   // scalar basic moments contribute directly
            for (int x = 0; x < nb; ++x)
                if (is_scalar[x]) {
                    Item it;
                    it.recs.push_back(make_rec(row[x], plan.one_row, 0, 0, 1.0));
                    it.recs.push_back(make_rec(plan.zero_row, plan.zero_row, plan.scratch_row,
                                               DAG_ENERGY | DAG_END, scal[x]));
                    it.energy = energy_index[x];
                    items.push_back(std::move(it));
                }
        }
        for (int x = nb; x < M; ++x) {
            if (!is_target[x] || level[x] != L)
                continue;
            if (!is_operand[x] && !is_scalar[x])
                continue;   // contributes nothing
            Item it;
            // rules of x with the same operand pair are one record with the
            // summed coefficient (first occurrence keeps its place)
            const auto &rl = rules_of[x];
            std::vector<std::pair<long, double>> terms;
            for (size_t k = 0; k < rl.size(); ++k) {
                const int *r = &m.times[4 * rl[k]];
                const long key = (long)std::min(r[0], r[1]) * M + std::max(r[0], r[1]);
                auto hit = std::find_if(terms.begin(), terms.end(),
                                        [&](const auto &t) { return t.first == key; });
                if (hit == terms.end())
                    terms.push_back({key, (double)r[2]});
                else
                    hit->second += (double)r[2];
            }
            for (const auto &t : terms)
                it.recs.push_back(make_rec(row[(int)(t.first / M)], row[(int)(t.first % M)], 0, 0,
                                           t.second));
            // the item ends with its energy term (scalars) and the store of
            // the product moment (operands; otherwise a scratch row)
            const int out = is_operand[x] ? row[x] : plan.scratch_row;
            if (is_scalar[x]) {
                it.recs.push_back(make_rec(plan.zero_row, plan.zero_row, out,
                                           DAG_ENERGY | DAG_END, scal[x]));
                it.energy = energy_index[x];
            }
            else
                it.recs.back().outf = (unsigned)out | ((unsigned)DAG_END << 16);
            items.push_back(std::move(it));
        }
        nfwd_phases += emit_phase(items, plan, pool);
    }
    plan.n_fwd = nfwd_phases;

    // ---- reverse phases ----------------------------------------------------
    // uses of each operand: (target, other operand, coefficient)
    struct Use {
        int target, other;
        double c;
    };
    // Uses with the same (target, other operand) are one term with the summed
    // coefficient: the two adjoint terms c adj_t m_a of a square m_a m_a, and
    // repeated rules of one target and pair.
    std::vector<std::vector<Use>> uses(M);
    auto add_use = [&](int x, int target, int other, double c) {
        for (Use &u : uses[x])
            if (u.target == target && u.other == other) {
                u.c += c;
                return;
            }
        uses[x].push_back({target, other, c});
    };
    for (int t = 0; t < T; ++t) {
        const int *r = &m.times[4 * t];
        add_use(r[0], r[3], r[1], (double)r[2]);
        add_use(r[1], r[3], r[0], (double)r[2]);
    }
    auto make_item = [&](int x, int out, unsigned flags) {
        Item it;
        if (scal[x] != 0.0)   // acc starts at the scalar coefficient of x
            it.recs.push_back(make_rec(plan.one_row, plan.one_row, 0, 0, scal[x]));
        for (const Use &u : uses[x]) {
            if (adjrow[u.target] >= 0)
                it.recs.push_back(make_rec(adjrow[u.target], row[u.other], 0, 0, u.c));
            else if (is_scalar[u.target])
                it.recs.push_back(make_rec(plan.one_row, row[u.other], 0, 0, u.c * scal[u.target]));
        }
        if (it.recs.empty())
            it.recs.push_back(make_rec(plan.zero_row, plan.zero_row, 0, 0, 0.0));
        const unsigned old = it.recs.back().outf >> 16;
        it.recs.back().outf = (unsigned)out | ((old | DAG_END | flags) << 16);
        return it;
    };
    int nrev = 0;
    for (int L = maxlevel - 1; L >= 1; --L) {
        std::vector<Item> items;
        for (int x = nb; x < M; ++x)
            if (adjrow[x] >= 0 && level[x] == L)
                items.push_back(make_item(x, adjrow[x], 0));
        nrev += emit_phase(items, plan, pool);
    }
    {
        std::vector<Item> items;
        std::vector<char> slot_used(nslot, 0);
        for (int x = 0; x < nb; ++x) {
            items.push_back(make_item(x, slot_of_basic[x], DAG_GLOBAL));
            slot_used[slot_of_basic[x]] = 1;
        }
        for (int s = 0; s < nslot; ++s)
            if (!slot_used[s]) {
                Item it;
                it.recs.push_back(make_rec(plan.zero_row, plan.zero_row, s,
                                           DAG_END | DAG_GLOBAL, 0.0));
                items.push_back(std::move(it));
            }
        nrev += emit_phase(items, plan, pool);
    }
    plan.n_rev = nrev;
    if (plan.nrows >= 65535 || (int)plan.phase_rows.size() > DAG_MAX_PHASES) {
        if (err)
            *err = "moment graph too large (" + std::to_string(plan.nrows) + " rows, " +
                   std::to_string(plan.phase_rows.size()) + " phases)";
        return false;
    }
    return true;
}

// The record program on 32 and on 64 streams; 64 streams (16 warps per block)
// run a padded record slot about 10% faster (level-20 graph: 14.6 ms for 15.1k
// slots against 15.7 ms for 14.6k on 32), so they are kept unless their padding
// costs more than that.
bool build_dag_plan(const ModelHost &m, int shape, const std::vector<int> &slot_of_basic,
                    DagPlan &plan, std::string *err)
{
    DagPlan p32, p64;
    if (!build_dag_plan_streams(m, shape, slot_of_basic, DAG_STREAMS, p32, err))
        return false;
    if (!build_dag_plan_streams(m, shape, slot_of_basic, DAG_STREAMS_LARGE, p64, err))
        return false;
    plan = 0.9 * (double)p64.recs.size() < (double)p32.recs.size() ? std::move(p64)
                                                                     : std::move(p32);
    return true;
}

// Eigen's fixed-size 3x3 inverse in its own operation order (the order the
// reference's Atoms::cell_.inverse() rounds in, base/neighborhoods_base.h:
// 113-126): det = (c0*m00 + c1*m10) + c2*m20, inv(i,j) = cofactor(j,i) * (1/det).
static double cof3(const double *m, int i, int j)
{
    int i1 = (i + 1) % 3, i2 = (i + 2) % 3, j1 = (j + 1) % 3, j2 = (j + 2) % 3;
    return m[i1 * 3 + j1] * m[i2 * 3 + j2] - m[i1 * 3 + j2] * m[i2 * 3 + j1];
}

bool prepare_struct(const double *cell, const int *pbc, double cutoff, NbStruct &out,
                    std::string *error)
{
    for (int a = 0; a < 3; ++a)
        if (pbc && !pbc[a]) {
            if (error)
                *error = "the GPU neighbour builder handles fully periodic cells; pass "
                         "explicit neighbour lists (mtpb_efs_csr) for other boundaries";
            return false;
        }
    for (int i = 0; i < 9; ++i) {
        if (!std::isfinite(cell[i])) {
            if (error)
                *error = "cell must be finite";
            return false;
        }
        out.cell[i] = cell[i];
    }
    volatile double c0 = cof3(cell, 0, 0), c1 = cof3(cell, 1, 0), c2 = cof3(cell, 2, 0);
    volatile double det = (c0 * cell[0] + c1 * cell[3]) + c2 * cell[6];
    if (!(std::fabs(det) > 0)) {
        if (error)
            *error = "singular cell";
        return false;
    }
    const double invdet = 1.0 / det;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            out.inv[i * 3 + j] = cof3(cell, j, i) * invdet;
    // image basis (neighborhoods_base.h:36-48): rows sorted by squared norm,
    // stable for ties
    auto sqn = [&](int a) {
        const double *r = cell + 3 * a;
        return r[0] * r[0] + (r[1] * r[1] + r[2] * r[2]);
    };
    int axes[3] = {0, 1, 2};
    for (int i = 1; i < 3; ++i) {
        int v = axes[i], j = i;
        while (j > 0 && sqn(v) < sqn(axes[j - 1])) {
            axes[j] = axes[j - 1];
            --j;
        }
        axes[j] = v;
    }
    out.dims = 3;
    for (int k = 0; k < 3; ++k) {
        out.axes[k] = axes[k];
        for (int r = 0; r < 3; ++r)
            out.B[r][k] = cell[3 * axes[k] + r];
    }
    // cell grid: perpendicular widths V / |a_b x a_c|
    const double *rows[3] = {cell, cell + 3, cell + 6};
    double cr[3][3];
    for (int a = 0; a < 3; ++a) {
        const double *u = rows[(a + 1) % 3], *v = rows[(a + 2) % 3];
        cr[a][0] = u[1] * v[2] - u[2] * v[1];
        cr[a][1] = u[2] * v[0] - u[0] * v[2];
        cr[a][2] = u[0] * v[1] - u[1] * v[0];
    }
    const double vol =
        std::fabs(rows[0][0] * cr[0][0] + rows[0][1] * cr[0][1] + rows[0][2] * cr[0][2]);
    for (int a = 0; a < 3; ++a) {
        const double nrm = std::sqrt(cr[a][0] * cr[a][0] + cr[a][1] * cr[a][1] + cr[a][2] * cr[a][2]);
        const double width = vol / nrm;
        // cells at least rc thick (with a small safety margin)
        int n = (int)std::floor(width / (cutoff * (1.0 + 1e-9)));
        if (n < 1)
            n = 1;
        if (n > 1024)
            n = 1024;
        out.ncell[a] = n;
        const double thick = width / n;
        out.stencil[a] = (int)std::ceil(cutoff * (1.0 + 1e-9) / thick);
        if (out.stencil[a] > 64) {
            if (error)
                *error = "cell too thin for the cutoff (more than 64 periodic images)";
            return false;
        }
    }
    out.cutsq = cutoff * cutoff;
    out.cell0 = 0;
    return true;
}

} // namespace mtpb
