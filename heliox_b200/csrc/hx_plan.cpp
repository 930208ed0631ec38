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

std::string build_plan(const hx_group_desc& g, int nodes_per_pack, Plan& P) {
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

    // branch decomposition per cell (BFS over branches from the root)
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
    }

    // pack cells: LPT (largest first onto the least-loaded pack)
    long long total = n;
    int target = nodes_per_pack > 0 ? nodes_per_pack : 1024;
    int maxcell = *std::max_element(cell_size.begin(), cell_size.end());
    if (target < maxcell) target = maxcell;
    long long npack = (total + target - 1) / target;
    if (npack < 1) npack = 1;
    if (npack > ncell) npack = ncell;
    if (npack >= 148) npack = ((npack + 147) / 148) * 148;
    if (npack > ncell) npack = ncell;
    P.npack = (int)npack;
    std::vector<int> order(ncell);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return cell_size[x] > cell_size[y]; });
    std::vector<std::vector<int>> pack_cells(npack);
    {
        using E = std::pair<long long, int>;  // (load, pack)
        std::priority_queue<E, std::vector<E>, std::greater<E>> pq;
        for (int p = 0; p < npack; p++) pq.push({0, p});
        for (int c : order) {
            auto [ld, p] = pq.top();
            pq.pop();
            pack_cells[p].push_back(c);
            pq.push({ld + cell_size[c], p});
        }
        for (auto& v : pack_cells) std::sort(v.begin(), v.end());
    }

    // layout
    P.pack_node_off.assign(npack + 1, 0);
    P.pack_hh_off.assign(npack + 1, 0);
    P.pack_br_off.assign(npack + 1, 0);
    P.pack_lvl_off.assign(npack + 1, 0);
    P.pack_nlev.assign(npack, 0);
    P.gpu2ref.resize(n);
    P.ref2gpu.assign(n, -1);
    P.node_parent.resize(n);
    P.node_cell.resize(n);
    P.br_child_off.push_back(0);

    // density instance lookup by reference node
    std::vector<int> hh_of(n, -1), pas_of(n, -1);
    for (int j = 0; j < g.nhh; j++) hh_of[g.hh_node[j]] = j;
    for (int j = 0; j < g.npas; j++) pas_of[g.pas_node[j]] = j;
    std::vector<int> ic_cnt(n, 0);
    for (int j = 0; j < g.nic; j++) ic_cnt[g.ic_node[j]]++;
    std::vector<int> ic_first(n + 1, 0);
    for (int i = 0; i < n; i++) ic_first[i + 1] = ic_first[i] + ic_cnt[i];

    int gpos = 0;
    long long sum_nodes = 0;
    for (int p = 0; p < npack; p++) {
        // collect branches of the pack's cells, ordered by (level, cell, head)
        struct BRef {
            int c, b;
        };
        std::vector<BRef> brs;
        for (int c : pack_cells[p])
            for (int b = 0; b < (int)cbr[c].size(); b++) brs.push_back({c, b});
        std::stable_sort(brs.begin(), brs.end(), [&](const BRef& x, const BRef& y) {
            const Branch& X = cbr[x.c][x.b];
            const Branch& Y = cbr[y.c][y.b];
            if (X.level != Y.level) return X.level < Y.level;
            if (x.c != y.c) return x.c < y.c;
            return X.head_ref < Y.head_ref;
        });
        const int base = gpos;
        std::vector<int> ref2loc_local;  // filled via P.ref2gpu
        int nlev = 0;
        for (auto& r : brs) nlev = std::max(nlev, cbr[r.c][r.b].level + 1);
        P.pack_nlev[p] = nlev;
        // level offsets
        std::vector<int> lvl_off(nlev + 1, 0);
        for (auto& r : brs) lvl_off[cbr[r.c][r.b].level + 1]++;
        for (int L = 0; L < nlev; L++) lvl_off[L + 1] += lvl_off[L];
        for (int L = 0; L <= nlev; L++) P.level_br_off.push_back(lvl_off[L]);
        P.pack_lvl_off[p + 1] = P.pack_lvl_off[p] + nlev + 1;
        // assign node positions
        for (auto& r : brs) {
            const Branch& B = cbr[r.c][r.b];
            for (int ref : B.nodes) {
                P.gpu2ref[gpos] = ref;
                P.ref2gpu[ref] = gpos;
                P.node_cell[gpos] = r.c;
                gpos++;
            }
        }
        const int pn = gpos - base;
        sum_nodes += pn;
        // branches
        int crit = 0;
        std::vector<int> path_len(brs.size(), 0);
        for (size_t bi = 0; bi < brs.size(); bi++) {
            const Branch& B = cbr[brs[bi].c][brs[bi].b];
            P.br_head.push_back(P.ref2gpu[B.head_ref] - base);
            P.br_end.push_back(P.ref2gpu[B.end_ref] - base);
            int hp = g.parent[B.head_ref];
            P.br_parent.push_back(hp < 0 ? -1 : P.ref2gpu[hp] - base);
            // child heads of the branch end, descending reference index
            int e = B.end_ref;
            for (int k = child_off[e + 1] - 1; k >= child_off[e]; k--) P.br_child.push_back(P.ref2gpu[child[k]] - base);
            P.br_child_off.push_back((int)P.br_child.size());
        }
        // critical path (nodes on the longest root->leaf chain)
        {
            std::vector<int> depth(pn, 0);
            for (int l = 0; l < pn; l++) {
                int ref = P.gpu2ref[base + l];
                int pr = g.parent[ref];
                depth[l] = pr < 0 ? 1 : depth[P.ref2gpu[pr] - base] + 1;
                crit = std::max(crit, depth[l]);
            }
        }
        P.pack_br_off[p + 1] = P.pack_br_off[p] + (int)brs.size();
        P.pack_node_off[p + 1] = gpos;
        P.max_pack_nodes = std::max(P.max_pack_nodes, pn);
        P.max_levels = std::max(P.max_levels, nlev);
        P.max_crit = std::max(P.max_crit, crit);
    }
    P.imbalance = (double)P.max_pack_nodes / ((double)sum_nodes / (double)npack);

    // node parent / children in pack-local ids
    P.node_child_off.assign(n + 1, 0);
    for (int p = 0; p < npack; p++) {
        const int base = P.pack_node_off[p];
        for (int gi = base; gi < P.pack_node_off[p + 1]; gi++) {
            int ref = P.gpu2ref[gi];
            int pr = g.parent[ref];
            P.node_parent[gi] = pr < 0 ? -1 : P.ref2gpu[pr] - base;
            for (int k = child_off[ref]; k < child_off[ref + 1]; k++) P.node_child.push_back(P.ref2gpu[child[k]] - base);
            P.node_child_off[gi + 1] = (int)P.node_child.size();
        }
    }

    // mechanism instances in GPU order
    P.node_hh.assign(n, -1);
    P.node_pas.assign(n, -1);
    P.node_ic_off.assign(n + 1, 0);
    for (int p = 0; p < npack; p++) {
        int hh_local = 0;
        for (int gi = P.pack_node_off[p]; gi < P.pack_node_off[p + 1]; gi++) {
            int ref = P.gpu2ref[gi];
            if (hh_of[ref] >= 0) {
                P.node_hh[gi] = hh_local++;
                P.hh_gpu2ref.push_back(hh_of[ref]);
            }
            if (pas_of[ref] >= 0) {
                P.node_pas[gi] = (int)P.pas_gpu2ref.size();
                P.pas_gpu2ref.push_back(pas_of[ref]);
            }
            for (int k = ic_first[ref]; k < ic_first[ref + 1]; k++) {
                P.node_ic.push_back((int)P.ic_gpu2ref.size());
                P.ic_gpu2ref.push_back(k);
            }
            P.node_ic_off[gi + 1] = (int)P.node_ic.size();
        }
        P.pack_hh_off[p + 1] = P.pack_hh_off[p] + hh_local;
        P.max_pack_hh = std::max(P.max_pack_hh, hh_local);
    }
    if (P.br_child.empty()) P.br_child.push_back(0);
    if (P.node_child.empty()) P.node_child.push_back(0);
    if (P.node_ic.empty()) P.node_ic.push_back(0);
    return "";
}

void planned_solve_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed) {
    const double* A = transposed ? b : a;  // factor numerator (eliminates child into parent)
    const double* U = transposed ? a : b;  // coupling to the parent
    for (int p = 0; p < P.npack; p++) {
        const int base = P.pack_node_off[p];
        const int bbase = P.pack_br_off[p];
        const int* lo = &P.level_br_off[P.pack_lvl_off[p]];
        const int nlev = P.pack_nlev[p];
        double* dd = d + base;
        double* rr = rhs + base;
        const double* AA = A + base;
        const double* UU = U + base;
        for (int L = nlev - 1; L >= 0; L--) {
            for (int br = lo[L]; br < lo[L + 1]; br++) {
                const int gb = bbase + br;
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
            }
        }
        for (int L = 0; L < nlev; L++) {
            for (int br = lo[L]; br < lo[L + 1]; br++) {
                const int gb = bbase + br;
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
            }
        }
    }
}

}  // namespace hx
