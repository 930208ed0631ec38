// hx_plan.cpp -- see hx_plan.hpp.
#include "hx_plan.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <numeric>
#include <queue>
#include <sstream>

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

}  // namespace

std::string build_plan(const hx_group_desc& g, int nodes_per_warp, int max_pack_nodes, Plan& P) {
    std::string err = validate(g);
    if (!err.empty()) return err;
    P = Plan();
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
            while (nchild[cur] == 1) {
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

    // first-fit-decreasing packing of whole cells into CTAs by node count (the
    // shared-memory capacity; at most kWarpsPerCta cells), then the CTA's warps
    // are shared among its cells in proportion to their nodes (at least one
    // each, largest remainders first), so every thread of a CTA carries about
    // the same number of nodes.
    const int npw = nodes_per_warp > 0 ? nodes_per_warp : 144;
    const int maxcell = *std::max_element(cell_size.begin(), cell_size.end());
    int cap = npw * kWarpsPerCta;
    if (max_pack_nodes > 0) {
        if (maxcell > max_pack_nodes)
            return "a cell of " + std::to_string(maxcell) + " nodes exceeds the per-CTA capacity of " +
                   std::to_string(max_pack_nodes) + " nodes";
        cap = std::min(cap, max_pack_nodes);
    }
    cap = std::max(cap, maxcell);
    std::vector<int> wc(ncell, 1);
    std::vector<int> order(ncell);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return cell_size[x] > cell_size[y]; });
    std::vector<std::vector<int>> bins;
    std::vector<int> bin_n;
    for (int c : order) {
        int b = -1;
        for (int k = 0; k < (int)bins.size(); k++)
            if ((int)bins[k].size() < kWarpsPerCta && bin_n[k] + cell_size[c] <= cap) {
                b = k;
                break;
            }
        if (b < 0) {
            bins.push_back({});
            bin_n.push_back(0);
            b = (int)bins.size() - 1;
        }
        bins[b].push_back(c);
        bin_n[b] += cell_size[c];
    }
    for (size_t b = 0; b < bins.size(); b++) {
        const int nb = (int)bins[b].size();
        const double tot = (double)bin_n[b];
        int used = 0;
        std::vector<std::pair<double, int>> rem;
        for (int c : bins[b]) {
            const double share = kWarpsPerCta * (double)cell_size[c] / tot;
            wc[c] = std::max(1, (int)std::floor(share));
            used += wc[c];
            rem.push_back({share - std::floor(share), c});
        }
        // hand out the rest by largest remainder (then most nodes per warp)
        std::stable_sort(rem.begin(), rem.end(), [&](const std::pair<double, int>& x, const std::pair<double, int>& y) {
            return x.first > y.first;
        });
        for (size_t i = 0; used < kWarpsPerCta && nb > 0; i = (i + 1) % rem.size()) {
            wc[rem[i].second]++;
            used++;
        }
        // floor-at-one may have overshot for packs of many small cells: take warps
        // back from the cells with the fewest nodes per warp
        while (used > kWarpsPerCta) {
            int best = -1;
            double bv = 1e300;
            for (int c : bins[b]) {
                double v = (double)cell_size[c] / wc[c];
                if (wc[c] > 1 && v < bv) {
                    bv = v;
                    best = c;
                }
            }
            if (best < 0) break;
            wc[best]--;
            used--;
        }
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
            const std::vector<Branch>& B = cbr[c];
            P.cs_cell.push_back(c);
            P.cs_node0.push_back(gpos - base);
            P.cs_nnode.push_back(cell_size[c]);
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
                    P.node_cell[gpos] = c;
                    gpos++;
                }
        }
        // branches of the pack (cell by cell, already level-sorted)
        for (int c : bins[p])
            for (const Branch& br : cbr[c]) {
                P.br_head.push_back(P.ref2gpu[br.head_ref] - base);
                P.br_end.push_back(P.ref2gpu[br.end_ref] - base);
                int hp = g.parent[br.head_ref];
                P.br_parent.push_back(hp < 0 ? -1 : P.ref2gpu[hp] - base);
                int e = br.end_ref;
                for (int k = child_off[e + 1] - 1; k >= child_off[e]; k--)
                    P.br_child.push_back(P.ref2gpu[child[k]] - base);
                P.br_child_off.push_back((int)P.br_child.size());
            }
        const int pn = gpos - base;
        sum_nodes += pn;
        {
            std::vector<int> depth(pn, 0);
            for (int l = 0; l < pn; l++) {
                int pr = g.parent[P.gpu2ref[base + l]];
                depth[l] = pr < 0 ? 1 : depth[P.ref2gpu[pr] - base] + 1;
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
    if (P.node_child.empty()) P.node_child.push_back(0);
    if (P.node_ic.empty()) P.node_ic.push_back(0);
    return "";
}

// Replays the schedule: per pack, per cell slot, levels deepest-first then root-first.
template <class Tri, class Back>
static void walk_schedule(const Plan& P, Tri tri, Back back) {
    for (int p = 0; p < P.npack; p++) {
        const int base = P.pack_node_off[p];
        const int bbase = P.pack_br_off[p];
        for (int s = P.pack_slot_off[p]; s < P.pack_slot_off[p + 1]; s++) {
            const int* lo = &P.level_br_off[P.cs_lvl_off[s]];
            const int nlev = P.cs_nlev[s];
            for (int L = nlev - 1; L >= 0; L--)
                for (int br = lo[L]; br < lo[L + 1]; br++) tri(base, bbase + br);
            for (int L = 0; L < nlev; L++)
                for (int br = lo[L]; br < lo[L + 1]; br++) back(base, bbase + br);
        }
    }
}

void planned_solve_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed) {
    const double* A = transposed ? b : a;  // eliminates a child into its parent
    const double* U = transposed ? a : b;  // couples a node to its parent
    walk_schedule(
        P,
        [&](int base, int gb) {
            double* dd = d + base;
            double* rr = rhs + base;
            const double* AA = A + base;
            const double* UU = U + base;
            const int h = P.br_head[gb], e = P.br_end[gb];
            for (int k = P.br_child_off[gb]; k < P.br_child_off[gb + 1]; k++) {
                const int c = P.br_child[k];
                double f = AA[c] / dd[c];
                dd[e] -= f * UU[c];
                rr[e] -= f * rr[c];
            }
            for (int j = e; j > h; j--) {
                double f = AA[j] / dd[j];
                dd[j - 1] -= f * UU[j];
                rr[j - 1] -= f * rr[j];
            }
        },
        [&](int base, int gb) {
            double* dd = d + base;
            double* rr = rhs + base;
            const double* UU = U + base;
            const int h = P.br_head[gb], e = P.br_end[gb];
            const int par = P.br_parent[gb];
            if (par < 0) {
                rr[h] /= dd[h];
            } else {
                rr[h] -= UU[h] * rr[par];
                rr[h] /= dd[h];
            }
            for (int j = h + 1; j <= e; j++) {
                rr[j] -= UU[j] * rr[j - 1];
                rr[j] /= dd[j];
            }
        });
}

void planned_solve_pq_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed) {
    const double* A = transposed ? b : a;
    const double* U = transposed ? a : b;
    walk_schedule(
        P,
        [&](int base, int gb) {
            double* dd = d + base;
            double* rr = rhs + base;
            const double* AA = A + base;
            const double* UU = U + base;
            const int h = P.br_head[gb], e = P.br_end[gb];
            double de = dd[e], re = rr[e];
            for (int k = P.br_child_off[gb]; k < P.br_child_off[gb + 1]; k++) {
                const int c = P.br_child[k];
                de = std::fma(-(AA[c] * UU[c]), dd[c], de);
                re = std::fma(-AA[c], rr[c], re);
            }
            double pp = de, qq = 1.0, yy = re;
            for (int j = e; j > h; j--) {
                const double pn = std::fma(dd[j - 1], pp, -((AA[j] * UU[j]) * qq));
                const double yn = std::fma(rr[j - 1], pp, -(AA[j] * yy));
                const double ip = 1.0 / pp;
                dd[j] = qq * ip;
                rr[j] = yy * ip;
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
            dd[h] = qq * ip;
            rr[h] = yy * ip;
        },
        [&](int base, int gb) {
            double* dd = d + base;
            double* rr = rhs + base;
            const double* UU = U + base;
            const int h = P.br_head[gb], e = P.br_end[gb];
            const int par = P.br_parent[gb];
            double x = rr[h];
            if (par >= 0) x = std::fma(-(UU[h] * dd[h]), rr[par], x);
            rr[h] = x;
            for (int j = h + 1; j <= e; j++) {
                x = std::fma(-(UU[j] * dd[j]), x, rr[j]);
                rr[j] = x;
            }
        });
}

}  // namespace hx
