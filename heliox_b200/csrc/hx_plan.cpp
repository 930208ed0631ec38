// hx_plan.cpp -- see hx_plan.hpp.
#include "hx_plan.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <numeric>
#include <map>
#include <queue>
#include <random>
#include <set>
#include <sstream>
#include <unordered_map>

namespace hx {

namespace {

struct Branch {
    int head_ref, end_ref;  // reference node ids
    int parent_branch;      // index into the cell's branch list, -1 for the root branch
    int level;
    std::vector<int> nodes; // reference ids head..end
};

std::string validate(const hx_group_desc& g) {
    std::ostringstream e;
    if (g.ncell <= 0 || g.nnode < g.ncell) return "bad ncell/nnode";
    if (!g.parent || !g.a || !g.b || !g.area || !g.cm) return "missing node arrays";
    if (!(g.dt > 0)) return "dt must be positive";
    for (int i = 0; i < g.ncell; i++)
        if (g.parent[i] != -1) return "roots (first ncell nodes) must have parent -1";
    for (int i = g.ncell; i < g.nnode; i++)
        if (g.parent[i] < 0 || g.parent[i] >= i) {
            e << "parent[" << i << "]=" << g.parent[i] << " violates 0 <= parent < i";
            return e.str();
        }
    for (int i = 0; i < g.nnode; i++)
        if (!(g.area[i] > 0)) return "area must be positive";
    auto chk = [&](int n, const int* nodes, bool density, const char* nm) -> std::string {
        if (n < 0) return std::string(nm) + ": negative count";
        if (n && !nodes) return std::string(nm) + ": missing node indices";
        for (int j = 0; j < n; j++) {
            if (nodes[j] < 0 || nodes[j] >= g.nnode) return std::string(nm) + ": node index out of range";
            if (j && nodes[j] < nodes[j - 1]) return std::string(nm) + ": node indices must be sorted";
            if (j && density && nodes[j] == nodes[j - 1])
                return std::string(nm) + ": two instances of a density mechanism on one node";
        }
        return "";
    };
    std::string r;
    if (!(r = chk(g.nhh, g.hh_node, true, "hh")).empty()) return r;
    if (g.nhh && (!g.hh_gnabar || !g.hh_gkbar || !g.hh_gl || !g.hh_el || !g.hh_ena || !g.hh_ek))
        return "hh: missing parameter arrays";
    if (!(r = chk(g.npas, g.pas_node, true, "pas")).empty()) return r;
    if (g.npas && (!g.pas_g || !g.pas_e)) return "pas: missing parameter arrays";
    if (!(r = chk(g.nic, g.ic_node, false, "IClamp")).empty()) return r;
    if (g.nic && (!g.ic_del || !g.ic_dur || !g.ic_amp)) return "IClamp: missing parameter arrays";
    return "";
}

// Splits one cell's branches into a top unit and subtree units of at most
// cap nodes each: starting from the root branch, the branch whose subtree is
// largest among those hanging off the top unit moves into it until every
// hanging subtree fits.  Branch levels and parent links are renumbered per unit.
std::string split_cell(const std::vector<Branch>& Bin, const std::vector<int>& parent_ref, int cap,
                       std::vector<std::vector<Branch>>& units) {
    // parent branches from the node structure (the branch list is sorted by
    // level and head, so parent indices recorded while building it are stale)
    std::vector<Branch> B = Bin;
    const int nb = (int)B.size();
    {
        std::unordered_map<int, int> br_of;
        for (int i = 0; i < nb; i++)
            for (int r : B[i].nodes) br_of[r] = i;
        for (int i = 0; i < nb; i++) {
            const int pr = parent_ref[B[i].head_ref];
            B[i].parent_branch = pr < 0 ? -1 : br_of[pr];
        }
    }
    std::vector<std::vector<int>> kids(nb);
    for (int i = 0; i < nb; i++)
        if (B[i].parent_branch >= 0) kids[B[i].parent_branch].push_back(i);
    std::vector<long long> sub(nb, 0);
    for (int i = nb - 1; i >= 0; i--) {  // sorted by level: children after parents
        sub[i] += (long long)B[i].nodes.size();
        if (B[i].parent_branch >= 0) sub[B[i].parent_branch] += sub[i];
    }
    std::vector<char> top(nb, 0);
    top[0] = 1;
    long long top_nodes = (long long)B[0].nodes.size();
    for (;;) {
        int worst = -1;
        for (int i = 1; i < nb; i++)
            if (!top[i] && top[B[i].parent_branch] && (worst < 0 || sub[i] > sub[worst])) worst = i;
        if (worst < 0 || sub[worst] <= cap) break;
        top[worst] = 1;
        top_nodes += (long long)B[worst].nodes.size();
        if (top_nodes > cap) return "cell too large to split into CTA-sized parts";
    }
    units.clear();
    auto emit = [&](const std::vector<int>& members) {
        std::vector<Branch> U;
        std::vector<int> local(nb, -1);
        for (int i : members) {
            Branch br = B[i];
            const int pb = B[i].parent_branch;
            br.parent_branch = (pb >= 0 && local[pb] >= 0) ? local[pb] : -1;
            br.level = br.parent_branch < 0 ? 0 : U[br.parent_branch].level + 1;
            local[i] = (int)U.size();
            U.push_back(std::move(br));
        }
        std::vector<int> idx(U.size());
        std::iota(idx.begin(), idx.end(), 0);
        std::stable_sort(idx.begin(), idx.end(), [&](int x, int y) {
            if (U[x].level != U[y].level) return U[x].level < U[y].level;
            return U[x].head_ref < U[y].head_ref;
        });
        std::vector<int> pos(U.size());
        for (size_t k = 0; k < idx.size(); k++) pos[idx[k]] = (int)k;
        std::vector<Branch> S;
        for (int k : idx) {
            Branch br = U[k];
            if (br.parent_branch >= 0) br.parent_branch = pos[br.parent_branch];
            S.push_back(std::move(br));
        }
        units.push_back(std::move(S));
    };
    std::vector<int> tm;
    for (int i = 0; i < nb; i++)
        if (top[i]) tm.push_back(i);
    emit(tm);
    for (int r = 1; r < nb; r++) {
        if (top[r] || !top[B[r].parent_branch]) continue;
        std::vector<int> m;  // the subtree of r in BFS order
        std::queue<int> q;
        q.push(r);
        while (!q.empty()) {
            int i = q.front();
            q.pop();
            m.push_back(i);
            for (int c : kids[i]) q.push(c);
        }
        emit(m);
    }
    return "";
}

}  // namespace

std::string build_plan(const hx_group_desc& g, int nodes_per_warp, int max_pack_nodes, Plan& P, int nsm,
                       int warps_per_cta) {
    const int kW = std::max(1, std::min(warps_per_cta, kWarpsPerCta));
    std::string err = validate(g);
    if (!err.empty()) return err;
    P = Plan();
    P.warps = kW;
    const int n = g.nnode, ncell = g.ncell;
    P.ncell = ncell;
    P.nnode = n;
    P.nhh = g.nhh;
    P.npas = g.npas;
    P.nic = g.nic;

    // cell of node, children lists (ascending reference index)
    std::vector<int> cell(n);
    std::vector<int> nchild(n, 0);
    for (int i = 0; i < ncell; i++) cell[i] = i;
    for (int i = ncell; i < n; i++) {
        cell[i] = cell[g.parent[i]];
        nchild[g.parent[i]]++;
    }
    std::vector<int> child_off(n + 1, 0);
    for (int i = 0; i < n; i++) child_off[i + 1] = child_off[i] + nchild[i];
    std::vector<int> child(std::max(child_off[n], 1));
    {
        std::vector<int> fill(child_off.begin(), child_off.end() - 1);
        for (int i = ncell; i < n; i++) child[fill[g.parent[i]]++] = i;
    }
    std::vector<int> cell_size(ncell, 0);
    for (int i = 0; i < n; i++) cell_size[cell[i]]++;

    // branch decomposition per cell (BFS over branches from the root), then
    // branches sorted by (level, head reference index)
    std::vector<std::vector<Branch>> cbr(ncell);
    for (int c = 0; c < ncell; c++) {
        std::vector<Branch>& B = cbr[c];
        std::queue<std::pair<int, int>> q;  // (head ref, parent branch)
        q.push({c, -1});
        while (!q.empty()) {
            auto [h, pb] = q.front();
            q.pop();
            Branch br;
            br.head_ref = h;
            br.parent_branch = pb;
            br.level = pb < 0 ? 0 : B[pb].level + 1;
            int cur = h;
            br.nodes.push_back(cur);
            // an unbranched chain longer than kSegMax is cut into segments
            // (each a branch whose one child is the next segment)
            while (nchild[cur] == 1 && (int)br.nodes.size() < kSegMax) {
                cur = child[child_off[cur]];
                br.nodes.push_back(cur);
            }
            br.end_ref = cur;
            B.push_back(std::move(br));
            int me = (int)B.size() - 1;
            for (int k = child_off[cur]; k < child_off[cur + 1]; k++) q.push({child[k], me});
        }
        std::stable_sort(B.begin(), B.end(), [](const Branch& x, const Branch& y) {
            if (x.level != y.level) return x.level < y.level;
            return x.head_ref < y.head_ref;
        });
    }

    // units: one per cell, unless a single cell exceeds the per-CTA capacity,
    // in which case it is split into a top unit (containing the root) and
    // subtree units hanging off it (see split_cell)
    std::vector<std::vector<Branch>> ubr;
    std::vector<int> usize, ucell;
    int top_unit = -1;
    {
        const int cap_guess = max_pack_nodes > 0 ? max_pack_nodes : 0;
        const int maxc = *std::max_element(cell_size.begin(), cell_size.end());
        if (cap_guess > 0 && maxc > cap_guess) {
            if (ncell != 1) return "a cell exceeds the per-CTA capacity; only a group of one cell can be split";
            std::string se = split_cell(cbr[0], std::vector<int>(g.parent, g.parent + n), cap_guess, ubr);
            if (!se.empty()) return se;
            top_unit = 0;
            for (auto& B : ubr) {
                int sz = 0;
                for (auto& br : B) sz += (int)br.nodes.size();
                usize.push_back(sz);
                ucell.push_back(0);
            }
        } else {
            ubr = cbr;
            usize = cell_size;
            for (int c = 0; c < ncell; c++) ucell.push_back(c);
        }
    }
    const int nunit = (int)ubr.size();

    // Whole cells are packed into CTAs (at most one cell a warp and the
    // shared-memory capacity in nodes each); the CTA's warps are then shared
    // among its cells in proportion to their nodes (at least one each, largest
    // remainders first), so every thread of a CTA carries about the same
    // number of nodes.
    //   nsm > 0 (and no explicit nodes_per_warp): one CTA per SM, as few waves
    //     as the capacity allows -- cells are dealt largest first to the least
    //     loaded of nsm * waves CTAs (LPT), so the CTAs of a wave finish together;
    //   otherwise: first-fit decreasing into CTAs of nodes_per_warp * warps
    //     (default 144 nodes per warp) nodes.
    const bool balanced = nodes_per_warp <= 0 && nsm > 0 && max_pack_nodes > 0;
    const int npw = nodes_per_warp > 0 ? nodes_per_warp : 144;
    const int maxcell = *std::max_element(usize.begin(), usize.end());
    int cap = balanced ? max_pack_nodes : npw * kW;
    if (max_pack_nodes > 0) {
        if (maxcell > max_pack_nodes)
            return "a cell of " + std::to_string(maxcell) + " nodes exceeds the per-CTA capacity of " +
                   std::to_string(max_pack_nodes) + " nodes";
        cap = std::min(cap, max_pack_nodes);
    }
    cap = std::max(cap, maxcell);
    std::vector<int> wc(nunit, 1);
    std::vector<int> order;
    for (int u = 0; u < nunit; u++)
        if (u != top_unit) order.push_back(u);
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return usize[x] > usize[y]; });
    std::vector<std::vector<int>> bins;
    std::vector<int> bin_n;
    if (top_unit >= 0) {  // the top unit has a CTA of its own (pack 0)
        bins.push_back({top_unit});
        bin_n.push_back(usize[top_unit]);
    }
    const int b0 = (int)bins.size();
    if (balanced && !order.empty()) {
        long long total = 0;
        for (int c : order) total += usize[c];
        const int avail = std::max(1, nsm - b0);
        // Waves: the step kernels are latency bound, so a wave of CTAs takes
        // about the same time whatever their fill; the fewest waves that hold
        // the cells win.  Start from the capacity bound and, for each wave
        // count, deal the cells largest first to the least loaded CTA (LPT,
        // balanced); at high fill LPT can leave every CTA with less room than
        // the remaining cells, so those are then packed best-fit decreasing
        // (the fullest CTA that still holds the cell) into the same CTAs.
        // Only when both leave a cell over does the plan take one more wave.
        // Two capacities: a soft one (91 % of the shared-memory bound, 4 % left
        // for fragmentation) under which LPT and the balancing below have
        // room to even out the CTAs' step times, and the hard bound itself,
        // used (with best-fit packing) only when it saves a wave.
        const long long per_wave_max = (long long)avail * (long long)cap;
        const int waves_min =
            (int)std::max<long long>(1, (total + per_wave_max - 1) / std::max<long long>(per_wave_max, 1));
        const int soft = std::max(maxcell, (int)(0.91 * cap));
        const long long per_wave_soft = (long long)avail * (long long)(0.96 * soft);
        const int waves_soft =
            (int)std::max<long long>(1, (total + per_wave_soft - 1) / std::max<long long>(per_wave_soft, 1));
        int waves = waves_min;
        if (waves_soft == waves_min) cap = soft;
        const size_t nbase = bins.size();
        for (;; waves++) {
            long long K = (long long)avail * waves;
            K = std::max<long long>(K, ((long long)order.size() + kW - 1) / kW);
            K = std::min<long long>(K, (long long)order.size());
            bins.resize(nbase);
            bin_n.resize(nbase);
            for (long long k = 0; k < K; k++) {
                bins.push_back({});
                bin_n.push_back(0);
            }
            auto fits = [&](int k, int c) { return (int)bins[k].size() < kW && bin_n[k] + usize[c] <= cap; };
            // LPT
            std::set<std::pair<long long, int>> load;  // (nodes, bin)
            for (long long k = 0; k < K; k++) load.insert({0, (int)(b0 + k)});
            std::vector<int> left;
            for (int c : order) {
                int b = -1;
                for (auto it = load.begin(); it != load.end(); ++it)
                    if (fits(it->second, c)) {
                        b = it->second;
                        load.erase(it);
                        break;
                    }
                if (b < 0) {
                    left.push_back(c);
                    continue;
                }
                bins[b].push_back(c);
                bin_n[b] += usize[c];
                if ((int)bins[b].size() < kW) load.insert({bin_n[b], b});
            }
            if (left.empty()) break;
            // best-fit decreasing from scratch into the same CTAs
            for (size_t k = nbase; k < bins.size(); k++) {
                bins[k].clear();
                bin_n[k] = 0;
            }
            left.clear();
            std::multiset<std::pair<long long, int>> room;  // (free nodes, bin)
            for (size_t k = nbase; k < bins.size(); k++) room.insert({(long long)cap, (int)k});
            for (int c : order) {
                auto it = room.lower_bound({(long long)usize[c], -1});
                if (it == room.end()) {
                    left.push_back(c);
                    continue;
                }
                const int b = it->second;
                room.erase(it);
                bins[b].push_back(c);
                bin_n[b] += usize[c];
                if ((int)bins[b].size() < kW) room.insert({(long long)cap - bin_n[b], b});
            }
            // repair: a cell left over goes into a CTA whose room a move of one
            // of its cells to another CTA (with room for that cell) makes enough
            std::vector<int> still;
            for (int c : left) {
                bool placed = false;
                for (size_t bi = nbase; bi < bins.size() && !placed; bi++) {
                    const int free_i = cap - bin_n[bi];
                    if ((int)bins[bi].size() > kW) continue;
                    for (size_t yi = 0; yi < bins[bi].size() && !placed; yi++) {
                        const int y = bins[bi][yi];
                        if (free_i + usize[y] < usize[c]) continue;
                        for (size_t bj = nbase; bj < bins.size(); bj++) {
                            if (bj == bi || cap - bin_n[bj] < usize[y] || (int)bins[bj].size() >= kW) continue;
                            bins[bj].push_back(y);
                            bin_n[bj] += usize[y];
                            bins[bi][yi] = c;
                            bin_n[bi] += usize[c] - usize[y];
                            placed = true;
                            break;
                        }
                    }
                }
                if (!placed) still.push_back(c);
            }
            left.swap(still);
            if (left.empty()) break;
            if (K >= (long long)order.size()) {  // one cell per CTA already: keep the rest in CTAs of their own
                for (int c : left) {
                    bins.push_back({c});
                    bin_n.push_back(usize[c]);
                }
                break;
            }
        }
        // bins left empty stay for the balancing below to fill; the ones still
        // empty after it are dropped there
    } else {
        for (int c : order) {
            int b = -1;
            for (int k = b0; k < (int)bins.size(); k++)
                if ((int)bins[k].size() < kW && bin_n[k] + usize[c] <= cap) {
                    b = k;
                    break;
                }
            if (b < 0) {
                bins.push_back({});
                bin_n.push_back(0);
                b = (int)bins.size() - 1;
            }
            bins[b].push_back(c);
            bin_n[b] += usize[c];
        }
    }
    // Warps per cell and (balanced mode) the choice of cells per CTA follow an
    // estimate of a cell's forward + backward step time with w warps: the
    // latency of its Hines solve plus the per-node loops, whose time goes with
    // the nodes each thread carries.  The reduced-tree solve (hines_rt) goes
    // with the longest segment times the segments a thread carries, plus the
    // number of segment levels.  The constants are least-squares fits of
    // per-cell clock64 timings of the forward + backward kernels on B200
    // (1024 config-2 cells, one wave; 2-3 % mean error); only their ratios
    // matter.  A CTA finishes with its slowest cell, so warps go one at a time
    // to the cell with the largest estimate, and in balanced mode cells are
    // moved / swapped out of the slowest CTA while that lowers its estimate.
    constexpr double kRtSeg = 662.0, kRtLevel = 2930.0, kRtIter = 10651.0;
    std::vector<double> uh_seg(nunit, 0.0), uh_lvl(nunit, 0.0);
    std::vector<int> useg(nunit, 0);
    for (int u = 0; u < nunit; u++) {
        std::set<int> levels;
        int maxseg = 0;
        for (const Branch& br : ubr[u]) {
            levels.insert(br.level);
            maxseg = std::max(maxseg, (int)br.nodes.size());
        }
        uh_seg[u] = kRtSeg * maxseg;
        uh_lvl[u] = kRtLevel * (double)levels.size();
        useg[u] = (int)ubr[u].size();
    }
    auto unit_time = [&](int u, int w) {
        const double it = std::ceil((double)usize[u] / (32.0 * (double)w));
        const double per_thread = std::ceil((double)useg[u] / (32.0 * (double)w));
        return uh_seg[u] * per_thread + uh_lvl[u] + kRtIter * it;
    };
    // greedy warps of one CTA; returns the CTA's estimate
    auto assign_warps = [&](const std::vector<int>& cs, std::vector<int>& w) {
        for (int c : cs) w[c] = 1;
        int used = (int)cs.size();
        while (used < kW && !cs.empty()) {
            int best = -1;
            double bt = -1.0;
            for (int c : cs) {
                const double t = unit_time(c, w[c]);
                if (t > bt && unit_time(c, w[c] + 1) < t) {
                    bt = t;
                    best = c;
                }
            }
            if (best < 0) {  // no cell gets faster: spread the rest by nodes per warp
                for (int c : cs)
                    if (best < 0 || (double)usize[c] / w[c] > (double)usize[best] / w[best]) best = c;
            }
            w[best]++;
            used++;
        }
        double t = 0.0;
        for (int c : cs) t = std::max(t, unit_time(c, w[c]));
        return t;
    };
    if (balanced && (int)bins.size() > b0 + 1) {
        std::vector<int> wtmp(nunit, 1);
        std::vector<double> bt(bins.size(), 0.0);
        for (size_t k = b0; k < bins.size(); k++) bt[k] = assign_warps(bins[k], wtmp);
        std::mt19937 rng(20240611u);
        const int nbin = (int)bins.size() - b0;
        const int iters = std::min(60000, 4000 + 40 * nbin);
        for (int it = 0; it < iters; it++) {
            int a = b0;
            for (int k = b0; k < (int)bins.size(); k++)
                if (bt[k] > bt[a]) a = k;
            const int o = b0 + (int)(rng() % (unsigned)nbin);
            if (o == a || bins[a].empty()) continue;
            const int ia = (int)(rng() % bins[a].size());
            const int ca = bins[a][ia];
            std::vector<int> na = bins[a], no = bins[o];
            int dn_a = -usize[ca], dn_o = usize[ca];
            na.erase(na.begin() + ia);
            const bool move = (rng() & 1) || bins[o].empty();
            if (move) {
                if (na.empty() || (int)no.size() >= kW) continue;
                no.push_back(ca);
            } else {
                const int io = (int)(rng() % bins[o].size());
                const int co = bins[o][io];
                no.erase(no.begin() + io);
                no.push_back(ca);
                na.push_back(co);
                dn_a += usize[co];
                dn_o -= usize[co];
            }
            if (bin_n[a] + dn_a > cap || bin_n[o] + dn_o > cap) continue;
            const double ta = assign_warps(na, wtmp), to = assign_warps(no, wtmp);
            if (std::max(ta, to) < bt[a]) {
                bins[a].swap(na);
                bins[o].swap(no);
                bin_n[a] += dn_a;
                bin_n[o] += dn_o;
                bt[a] = ta;
                bt[o] = to;
            }
        }
        std::vector<std::vector<int>> kept;
        std::vector<int> kept_n;
        for (size_t k = 0; k < bins.size(); k++)
            if (!bins[k].empty()) {
                kept.push_back(std::move(bins[k]));
                kept_n.push_back(bin_n[k]);
            }
        bins.swap(kept);
        bin_n.swap(kept_n);
    }
    P.est_max = 0.0;
    P.est_mean = 0.0;
    for (size_t b = 0; b < bins.size(); b++) {
        const double t = assign_warps(bins[b], wc);
        P.est_max = std::max(P.est_max, t);
        P.est_mean += t / (double)bins.size();
        std::sort(bins[b].begin(), bins[b].end());
    }
    const int npack = (int)bins.size();
    P.npack = npack;

    // layout
    P.pack_node_off.assign(npack + 1, 0);
    P.pack_slot_off.assign(npack + 1, 0);
    P.pack_br_off.assign(npack + 1, 0);
    P.pack_bch_off.assign(npack + 1, 0);
    P.pack_nch_off.assign(npack + 1, 0);
    P.gpu2ref.resize(n);
    P.ref2gpu.assign(n, -1);
    P.node_parent.resize(n);
    P.node_cell.resize(n);
    P.br_child_off.push_back(0);
    std::vector<int> ic_cnt(n, 0);
    for (int j = 0; j < g.nic; j++) ic_cnt[g.ic_node[j]]++;
    std::vector<int> ic_first(n + 1, 0);
    for (int i = 0; i < n; i++) ic_first[i + 1] = ic_first[i] + ic_cnt[i];

    int gpos = 0;
    long long sum_nodes = 0;
    for (int p = 0; p < npack; p++) {
        const int base = gpos;
        int wpos = 0, bar = 1, brl = 0;
        int pack_levels = 0, crit = 0;
        for (int c : bins[p]) {
            const std::vector<Branch>& B = ubr[c];
            P.cs_cell.push_back(ucell[c]);
            P.cs_node0.push_back(gpos - base);
            P.cs_nnode.push_back(usize[c]);
            P.cs_warp0.push_back(wpos);
            P.cs_nwarp.push_back(wc[c]);
            P.cs_bar.push_back(wc[c] > 1 ? bar++ : 0);
            wpos += wc[c];
            int nlev = B.back().level + 1;
            P.cs_lvl_off.push_back((int)P.level_br_off.size());
            P.cs_nlev.push_back(nlev);
            std::vector<int> lvl(nlev + 1, 0);
            for (const Branch& br : B) lvl[br.level + 1]++;
            for (int L = 0; L < nlev; L++) lvl[L + 1] += lvl[L];
            for (int L = 0; L <= nlev; L++) P.level_br_off.push_back(brl + lvl[L]);
            brl += (int)B.size();
            pack_levels = std::max(pack_levels, nlev);
            for (const Branch& br : B)
                for (int ref : br.nodes) {
                    P.gpu2ref[gpos] = ref;
                    P.ref2gpu[ref] = gpos;
                    P.node_cell[gpos] = ucell[c];
                    gpos++;
                }
        }
        // branches of the pack (cell by cell, already level-sorted); children
        // by head node and by pack-local branch id (-1: in another unit)
        {
            int pbr = 0;
            for (int c : bins[p]) {
                std::unordered_map<int, int> by_head;
                for (size_t k = 0; k < ubr[c].size(); k++) by_head[ubr[c][k].head_ref] = pbr + (int)k;
                for (const Branch& br : ubr[c]) {
                    P.br_head.push_back(P.ref2gpu[br.head_ref] - base);
                    P.br_end.push_back(P.ref2gpu[br.end_ref] - base);
                    int hp = g.parent[br.head_ref];
                    P.br_parent.push_back(hp < 0 ? -1 : P.ref2gpu[hp] - base);
                    int e = br.end_ref;
                    for (int k = child_off[e + 1] - 1; k >= child_off[e]; k--) {
                        P.br_child.push_back(P.ref2gpu[child[k]] - base);
                        auto it = by_head.find(child[k]);
                        P.br_child_br.push_back(it == by_head.end() ? -1 : it->second);
                    }
                    P.br_child_off.push_back((int)P.br_child.size());
                }
                pbr += (int)ubr[c].size();
            }
        }
        const int pn = gpos - base;
        sum_nodes += pn;
        {
            std::vector<int> depth(pn, 0);
            for (int l = 0; l < pn; l++) {
                int pr = g.parent[P.gpu2ref[base + l]];
                const int pl = pr < 0 ? -1 : P.ref2gpu[pr] - base;
                depth[l] = (pl < 0 || pl >= l) ? 1 : depth[pl] + 1;
                crit = std::max(crit, depth[l]);
            }
        }
        P.pack_slot_off[p + 1] = (int)P.cs_cell.size();
        P.pack_br_off[p + 1] = P.pack_br_off[p] + brl;
        P.pack_bch_off[p + 1] = (int)P.br_child.size();
        P.pack_node_off[p + 1] = gpos;
        // node parent / children (pack-local)
        for (int gi = base; gi < gpos; gi++) {
            int ref = P.gpu2ref[gi];
            int pr = g.parent[ref];
            P.node_parent[gi] = pr < 0 ? -1 : P.ref2gpu[pr] - base;
            for (int k = child_off[ref]; k < child_off[ref + 1]; k++) P.node_child.push_back(P.ref2gpu[child[k]] - base);
        }
        P.pack_nch_off[p + 1] = (int)P.node_child.size();
        P.max_pack_nodes = std::max(P.max_pack_nodes, pn);
        P.max_levels = std::max(P.max_levels, pack_levels);
        P.max_crit = std::max(P.max_crit, crit);
        P.max_pack_branches = std::max(P.max_pack_branches, brl);
        P.max_pack_bch = std::max(P.max_pack_bch, P.pack_bch_off[p + 1] - P.pack_bch_off[p]);
        P.max_pack_nch = std::max(P.max_pack_nch, P.pack_nch_off[p + 1] - P.pack_nch_off[p]);
    }
    P.imbalance = (double)P.max_pack_nodes / ((double)sum_nodes / (double)npack);
    if (top_unit >= 0) {
        // links between the top unit (pack 0) and the subtree units: the
        // subtree roots' parents, the top nodes' children and branch children
        // in other packs are written as -(2 + subtree id)
        std::vector<int> pack_of(n);
        for (int p = 0; p < npack; p++)
            for (int gi = P.pack_node_off[p]; gi < P.pack_node_off[p + 1]; gi++) pack_of[gi] = p;
        std::vector<int> sub_of_root(n, -1);
        for (int p = 1; p < npack; p++)
            for (int s2 = P.pack_slot_off[p]; s2 < P.pack_slot_off[p + 1]; s2++) {
                const int root = P.pack_node_off[p] + P.cs_node0[s2];
                const int id = (int)P.sub_root.size();
                sub_of_root[root] = id;
                P.sub_root.push_back(root);
                P.sub_parent.push_back(P.ref2gpu[g.parent[P.gpu2ref[root]]]);
            }
        P.nsub = (int)P.sub_root.size();
        auto code = [&](int gi_other, int p, int base) {
            return pack_of[gi_other] == p ? gi_other - base : -(2 + sub_of_root[gi_other]);
        };
        for (int p = 0; p < npack; p++) {
            const int base = P.pack_node_off[p];
            // a subtree root's parent link carries the subtree's own id
            for (int gi = base; gi < P.pack_node_off[p + 1]; gi++) {
                const int pr = g.parent[P.gpu2ref[gi]];
                if (pr >= 0)
                    P.node_parent[gi] = pack_of[P.ref2gpu[pr]] == p ? P.ref2gpu[pr] - base : -(2 + sub_of_root[gi]);
            }
            // children lists rebuilt in their original orders with final indices
            int k = P.pack_nch_off[p];
            for (int gi = base; gi < P.pack_node_off[p + 1]; gi++) {
                const int ref = P.gpu2ref[gi];
                for (int c = child_off[ref]; c < child_off[ref + 1]; c++) P.node_child[k++] = code(P.ref2gpu[child[c]], p, base);
            }
            for (int b = P.pack_br_off[p]; b < P.pack_br_off[p + 1]; b++) {
                const int hg = P.br_head[b] + base, hr = P.gpu2ref[hg];
                P.br_parent[b] = g.parent[hr] < 0 ? -1
                                 : pack_of[P.ref2gpu[g.parent[hr]]] == p ? P.ref2gpu[g.parent[hr]] - base
                                                                         : -(2 + sub_of_root[hg]);
                const int er = P.gpu2ref[P.br_end[b] + base];
                int kk = P.br_child_off[b];
                for (int c = child_off[er + 1] - 1; c >= child_off[er]; c--) P.br_child[kk++] = code(P.ref2gpu[child[c]], p, base);
            }
        }
    }
    P.node_child_off.assign(n + 1, 0);
    {
        int k = 0;
        for (int gi = 0; gi < n; gi++) {
            k += nchild[P.gpu2ref[gi]];
            P.node_child_off[gi + 1] = k;
        }
    }

    // mechanism instances
    std::vector<int> hh_of(n, -1), pas_of(n, -1);
    for (int j = 0; j < g.nhh; j++) hh_of[g.hh_node[j]] = j;
    for (int j = 0; j < g.npas; j++) pas_of[g.pas_node[j]] = j;
    P.node_hh.assign(n, -1);
    P.node_pas.assign(n, -1);
    P.node_ic_off.assign(n + 1, 0);
    for (int p = 0; p < npack; p++) {
        int hh_cnt = 0;
        for (int gi = P.pack_node_off[p]; gi < P.pack_node_off[p + 1]; gi++) {
            int ref = P.gpu2ref[gi];
            P.node_hh[gi] = hh_of[ref];
            P.node_pas[gi] = pas_of[ref];
            hh_cnt += hh_of[ref] >= 0;
            for (int k = ic_first[ref]; k < ic_first[ref + 1]; k++) {
                P.node_ic.push_back((int)P.ic_gpu2ref.size());
                P.ic_gpu2ref.push_back(k);
            }
            P.node_ic_off[gi + 1] = (int)P.node_ic.size();
        }
        P.max_pack_hh = std::max(P.max_pack_hh, hh_cnt);
    }
    if (P.br_child.empty()) P.br_child.push_back(0);
    if (P.br_child_br.empty()) P.br_child_br.push_back(-1);
    if (P.node_child.empty()) P.node_child.push_back(0);
    if (P.node_ic.empty()) P.node_ic.push_back(0);
    return "";
}

// Replays the schedule: per pack, per cell slot, levels deepest-first then
// root-first.  For a split cell the triangularisation visits the subtree
// packs before the top pack (pack 0) and the back-substitution the top pack
// first, as the kernels' grid barriers order them.
template <class Tri, class Back>
static void walk_schedule(const Plan& P, Tri tri, Back back) {
    auto run = [&](int p, bool do_tri) {
        const int base = P.pack_node_off[p];
        const int bbase = P.pack_br_off[p];
        for (int s = P.pack_slot_off[p]; s < P.pack_slot_off[p + 1]; s++) {
            const int* lo = &P.level_br_off[P.cs_lvl_off[s]];
            const int nlev = P.cs_nlev[s];
            if (do_tri) {
                for (int L = nlev - 1; L >= 0; L--)
                    for (int br = lo[L]; br < lo[L + 1]; br++) tri(base, bbase + br);
            } else {
                for (int L = 0; L < nlev; L++)
                    for (int br = lo[L]; br < lo[L + 1]; br++) back(base, bbase + br);
            }
        }
    };
    if (P.nsub > 0) {
        for (int p = P.npack - 1; p >= 0; p--) run(p, true);
        for (int p = 0; p < P.npack; p++) run(p, false);
        return;
    }
    for (int p = 0; p < P.npack; p++) {
        run(p, true);
        run(p, false);
    }
}

// global GPU index of a branch child / branch parent entry (codes of a split cell)
static inline int child_global(const Plan& P, int base, int c) { return c >= 0 ? base + c : P.sub_root[-c - 2]; }
static inline int parent_global(const Plan& P, int base, int c) {
    return c >= 0 ? base + c : (c == -1 ? -1 : P.sub_parent[-c - 2]);
}

void planned_solve_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed) {
    const double* A = transposed ? b : a;  // eliminates a child into its parent
    const double* U = transposed ? a : b;  // couples a node to its parent
    walk_schedule(
        P,
        [&](int base, int gb) {
            const int h = base + P.br_head[gb], e = base + P.br_end[gb];
            // children of the end node, descending reference index
            for (int k = P.br_child_off[gb]; k < P.br_child_off[gb + 1]; k++) {
                const int c = child_global(P, base, P.br_child[k]);
                double pp = A[c] / d[c];
                d[e] -= pp * U[c];
                rhs[e] -= pp * rhs[c];
            }
            for (int j = e; j > h; j--) {
                double pp = A[j] / d[j];
                d[j - 1] -= pp * U[j];
                rhs[j - 1] -= pp * rhs[j];
            }
        },
        [&](int base, int gb) {
            const int h = base + P.br_head[gb], e = base + P.br_end[gb];
            const int par = parent_global(P, base, P.br_parent[gb]);
            if (par >= 0) rhs[h] -= U[h] * rhs[par];
            rhs[h] /= d[h];
            for (int j = h + 1; j <= e; j++) {
                rhs[j] -= U[j] * rhs[j - 1];
                rhs[j] /= d[j];
            }
        });
}

void planned_solve_pq_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed) {
    const double* A = transposed ? b : a;
    const double* U = transposed ? a : b;
    walk_schedule(
        P,
        [&](int base, int gb) {
            const int h = base + P.br_head[gb], e = base + P.br_end[gb];
            double de = d[e], re = rhs[e];
            for (int k = P.br_child_off[gb]; k < P.br_child_off[gb + 1]; k++) {
                const int c = child_global(P, base, P.br_child[k]);
                de = std::fma(-(A[c] * U[c]), d[c], de);
                re = std::fma(-A[c], rhs[c], re);
            }
            double pp = de, qq = 1.0, yy = re;
            for (int j = e; j > h; j--) {
                const double pn = std::fma(d[j - 1], pp, -((A[j] * U[j]) * qq));
                const double yn = std::fma(-A[j], yy, rhs[j - 1] * pp);
                const double ip = 1.0 / pp;
                d[j] = qq * ip;
                rhs[j] = yy * ip;
                qq = pp;
                pp = pn;
                yy = yn;
                if (((e - j) & 3) == 3) {
                    const double s = std::ldexp(1.0, -std::ilogb(pp));
                    pp *= s;
                    qq *= s;
                    yy *= s;
                }
            }
            const double ip = 1.0 / pp;
            d[h] = qq * ip;
            rhs[h] = yy * ip;
        },
        [&](int base, int gb) {
            const int h = base + P.br_head[gb], e = base + P.br_end[gb];
            const int par = parent_global(P, base, P.br_parent[gb]);
            double x = rhs[h];
            if (par >= 0) x = std::fma(-(U[h] * d[h]), rhs[par], x);
            rhs[h] = x;
            for (int j = h + 1; j <= e; j++) {
                x = std::fma(-(U[j] * d[j]), x, rhs[j]);
                rhs[j] = x;
            }
        });
}

void planned_solve_rt_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed) {
    const double* A = transposed ? b : a;
    const double* U = transposed ? a : b;
    std::vector<double> cd(P.br_head.size(), 0.0), cr(P.br_head.size(), 0.0), Fe(P.br_head.size(), 0.0),
        Ge(P.br_head.size(), 0.0);
    for (int p = 0; p < P.npack; p++) {
        const int base = P.pack_node_off[p];
        const int bbase = P.pack_br_off[p];
        for (int sl = P.pack_slot_off[p]; sl < P.pack_slot_off[p + 1]; sl++) {
            const int* lo = &P.level_br_off[P.cs_lvl_off[sl]];
            const int nlev = P.cs_nlev[sl];
            auto H = [&](int br) { return base + P.br_head[bbase + br]; };
            auto E = [&](int br) { return base + P.br_end[bbase + br]; };
            auto PP = [&](int br) { const int v = P.br_parent[bbase + br]; return v < 0 ? -1 : base + v; };
            // 1. segment interiors, top-down
            for (int br = lo[0]; br < lo[nlev]; br++) {
                const int h = H(br), e = E(br), gb = bbase + br;
                if (h == e) {
                    Fe[gb] = A[h];
                    Ge[gb] = U[h];
                    cd[gb] = cr[gb] = 0.0;
                    continue;
                }
                double inv = 1.0 / d[h], rp = rhs[h], F = A[h], G = U[h];
                double dD = F * G * inv, dR = F * rp * inv;
                d[h] = inv;
                for (int k = h + 1; k < e; k++) {
                    const double Dk = std::fma(-(U[k] * A[k]), inv, d[k]);
                    const double rk = std::fma(-(U[k] * rp), inv, rhs[k]);
                    F = -(F * A[k]) * inv;
                    G = -(U[k] * G) * inv;
                    inv = 1.0 / Dk;
                    rp = rk;
                    dD = std::fma(F * G, inv, dD);
                    dR = std::fma(F * rp, inv, dR);
                    d[k] = inv;
                }
                d[e] = std::fma(-(U[e] * A[e]), inv, d[e]);
                rhs[e] = std::fma(-(U[e] * rp), inv, rhs[e]);
                Fe[gb] = -(F * A[e]) * inv;
                Ge[gb] = -(U[e] * G) * inv;
                cd[gb] = dD;
                cr[gb] = dR;
            }
            // 2. tree of segment ends
            for (int L = nlev - 1; L >= 0; L--)
                for (int br = lo[L]; br < lo[L + 1]; br++) {
                    const int e = E(br), gb = bbase + br;
                    double De = d[e], Re = rhs[e];
                    for (int k = P.br_child_off[gb]; k < P.br_child_off[gb + 1]; k++) {
                        const int c = bbase + P.br_child_br[k];
                        De -= cd[c];
                        Re -= cr[c];
                    }
                    const double ie = 1.0 / De, ge = Re * ie, he = Ge[gb] * ie;
                    cd[gb] = std::fma(Fe[gb], he, cd[gb]);
                    cr[gb] = std::fma(Fe[gb], ge, cr[gb]);
                    d[e] = he;
                    rhs[e] = ge;
                }
            for (int L = 0; L < nlev; L++)
                for (int br = lo[L]; br < lo[L + 1]; br++) {
                    const int e = E(br), par = PP(br);
                    double x = rhs[e];
                    if (par >= 0) x = std::fma(-d[e], rhs[par], x);
                    rhs[e] = x;
                }
            // 3. interiors
            for (int br = lo[0]; br < lo[nlev]; br++) {
                const int h = H(br), e = E(br), par = PP(br);
                if (h == e) continue;
                double t = rhs[h];
                if (par >= 0) t = std::fma(-U[h], rhs[par], t);
                t *= d[h];
                rhs[h] = t;
                for (int k = h + 1; k < e; k++) {
                    t = std::fma(-(U[k] * d[k]), t, rhs[k] * d[k]);
                    rhs[k] = t;
                }
                double x = rhs[e];
                for (int k = e - 1; k >= h; k--) {
                    x = std::fma(-(A[k + 1] * d[k]), x, rhs[k]);
                    rhs[k] = x;
                }
            }
        }
    }
}

}  // namespace hx
