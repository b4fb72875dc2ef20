// Expert parallelism by all-to-all: the host plan of one step.
//
// Each of `world` ranks holds its own tokens and experts [ne r / world,
// ne (r + 1) / world). After every rank routed its tokens, each (token,
// choice) row goes to the rank holding its expert (dispatch), that rank runs
// its experts over the rows it received, and every result row goes back to
// the token's rank (combine), where the choice-order sum runs as on one GPU.
// This plan is what one rank needs, computed on the host from every rank's
// chosen experts (which the ranks exchange first): what it sends where, what
// it receives from whom, and the dispatch of the received rows over its own
// experts -- grouped by expert, ascending row within one, chunks of at most
// nt rows, as the router's own dispatch lays out its slots
// (moe.cuh moe_dispatch). Host code only (no CUDA).
#pragma once

#include <vector>

namespace sb {

struct MoeA2aPlan {
    // rows this rank sends, grouped by destination rank, (token, choice) order within one
    std::vector<int> send_tok;          // the token row to send
    std::vector<int> send_slot;         // its slot token * k + choice (where its result lands)
    std::vector<int> send_cnt, send_off;   // [world]
    // rows this rank receives, grouped by source rank, (token, choice) order within one
    std::vector<int> recv_cnt, recv_off;   // [world]
    std::vector<int> recv_exp;          // the expert of each received row
    // dispatch of the received rows (row index = slot) over this rank's experts
    std::vector<int> slots, ch_e, ch_s0, ch_n;
    int distinct = 0;
};

// The rank holding expert e of ne spread over world ranks.
inline int moe_owner(int e, int ne, int world) {
    int r = (int) ((long) e * world / ne);
    while (r + 1 < world && (long) ne * (r + 1) / world <= e) r++;
    while (r > 0 && (long) ne * r / world > e) r--;
    return r;
}

// n_tok[r]: rank r's tokens; sel[r]: its chosen experts [n_tok[r]][k].
// False if an expert id is out of range.
inline bool moe_a2a_plan(int world, int rank, int ne, int k, int nt, const int * n_tok, const int * const * sel,
                         MoeA2aPlan & p) {
    p = MoeA2aPlan();
    p.send_cnt.assign(world, 0);
    p.send_off.assign(world, 0);
    p.recv_cnt.assign(world, 0);
    p.recv_off.assign(world, 0);
    const int T = n_tok[rank];
    for (int d = 0, off = 0; d < world; d++) {
        p.send_off[d] = off;
        for (int t = 0; t < T; t++)
            for (int j = 0; j < k; j++) {
                const int e = sel[rank][t * k + j];
                if (e < 0 || e >= ne) return false;
                if (moe_owner(e, ne, world) != d) continue;
                p.send_tok.push_back(t);
                p.send_slot.push_back(t * k + j);
                p.send_cnt[d]++;
            }
        off += p.send_cnt[d];
    }
    for (int r = 0, off = 0; r < world; r++) {
        p.recv_off[r] = off;
        for (int t = 0; t < n_tok[r]; t++)
            for (int j = 0; j < k; j++) {
                const int e = sel[r][t * k + j];
                if (e < 0 || e >= ne) return false;
                if (moe_owner(e, ne, world) != rank) continue;
                p.recv_exp.push_back(e);
                p.recv_cnt[r]++;
            }
        off += p.recv_cnt[r];
    }
    // received rows grouped by expert, ascending within one, chunks of nt
    std::vector<std::vector<int>> by(ne);
    for (int i = 0; i < (int) p.recv_exp.size(); i++) by[p.recv_exp[i]].push_back(i);
    for (int e = 0; e < ne; e++) {
        if (by[e].empty()) continue;
        p.distinct++;
        const int s0 = (int) p.slots.size();
        p.slots.insert(p.slots.end(), by[e].begin(), by[e].end());
        for (int c = 0; c * nt < (int) by[e].size(); c++) {
            p.ch_e.push_back(e);
            p.ch_s0.push_back(s0 + c * nt);
            const int left = (int) by[e].size() - c * nt;
            p.ch_n.push_back(left < nt ? left : nt);
        }
    }
    return true;
}

}  // namespace sb
