// hx_netstim.cpp -- NetStim spike trains (host side of the event path).
//
// A NetStim's spikes do not depend on any membrane voltage, so the runtime
// generates the whole train of every NetStim once per forward length and
// routes it into the device event buckets before the first window.  The
// semantics are the reference's (src/spike/netstim.cpp:120-330 with the
// receive loop of Simulate::network_spike_receive_cpu, src/simulate.cpp:
// 916-941, and the self-event queue order of src/spike/spike.h:113-136):
//
//  * initialize: every instance with start >= 0 and number > 0 is switched on
//    and schedules an INIT event at max(0, start + invl - interval (1-noise));
//  * deliveries happen once at finitialize (t = 0) and at the start of every
//    step (t = t_k), for all queued events with time <= t + dt/2, batch by
//    batch until a batch schedules nothing more;
//  * INIT (instance on): init_sequence (every instance with number > 0 is
//    reset: on, ispike = 0) and a SELF event at t;
//  * SELF (instance on): ispike += 1, a spike at t, next_invl, and while still
//    on a SELF event at t + event.
//
// All NetStims share one Random123 stream (nrnran123, utils/nrnran123.cpp:
// 108-140).  next_invl redraws the interval of every instance with
// number > 0 and noise != 0, but only the firing instance's new interval is
// ever read, so its draw is taken directly by index: the d-th draw of the
// stream is word d % 4 of Philox4x32-10 at counter d / 4 (block 0 is all
// zeros in the reference's CPU mode, whose state is zero-initialised).
// Likewise init_sequence is applied lazily through a reset epoch.
#include "hx_netstim.hpp"

#include <cmath>
#include <cstdint>
#include <queue>
#include <vector>

namespace hx {

namespace {

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC11), key 0 (the global index nrnran123 leaves at 0).
void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t out[4]) {
    uint32_t k0 = 0, k1 = 0;
    for (int r = 0; r < 10; r++) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c0 = n0;
        c1 = (uint32_t)p1;
        c2 = n2;
        c3 = (uint32_t)p0;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

struct Stream {
    int mode;
    uint64_t cached_block = ~0ull;
    uint32_t r[4] = {0, 0, 0, 0};
    double negexp(uint64_t d) {
        const uint64_t b = d >> 2;
        if (b != cached_block) {
            if (mode == 0 && b == 0) {
                r[0] = r[1] = r[2] = r[3] = 0;
            } else {
                philox4x32_10((uint32_t)b, (uint32_t)(b >> 32), 0, 0, r);
            }
            cached_block = b;
        }
        static const double kShift32 = 1.0 / 4294967297.0;  // nrnran123_dblpick
        const double u = ((double)r[d & 3] + 1.0) * kShift32;
        return -std::log(u);
    }
};

enum { kSelf = 1, kInit = 2 };

struct Ev {
    double t;
    int id, flag;
};

// the spike buffer's comparator (spike.h:113-136) for one mechanism's self events
struct Later {
    bool operator()(const Ev& a, const Ev& b) const {
        if (std::fabs(a.t - b.t) > 1e-9) return a.t > b.t;
        return a.id > b.id;
    }
};

}  // namespace

void netstim_trains(const NetStimTable& ns, const std::vector<double>& tstart, double dt, int nstep,
                    std::vector<int>& out_id, std::vector<int>& out_step) {
    out_id.clear();
    out_step.clear();
    const int n = ns.n;
    if (n <= 0) return;
    std::vector<double> noise(n), on(n, 0.0), ispike(n, 0.0);
    std::vector<long long> epoch(n, 0);
    std::vector<long long> rank(n, -1);
    long long reset_epoch = 0, M = 0;
    Stream rng{ns.rng_mode};
    uint64_t draws = 0;
    for (int i = 0; i < n; i++) {
        double z = ns.noise[i];
        if (z < 0.0) z = 0.0;
        if (z > 1.0) z = 1.0;
        noise[i] = z;
    }
    for (int i = 0; i < n; i++)
        if (ns.number[i] > 0 && noise[i] != 0) rank[i] = M++;
    auto interval_of = [&](int i) { return ns.interval[i] <= 0.0 ? 0.01 : ns.interval[i]; };
    // lazily applied init_sequence: instances with number > 0 whose epoch is stale are (on, ispike 0)
    auto touch = [&](int i) {
        if (epoch[i] < reset_epoch) {
            if (ns.number[i] > 0) {
                on[i] = 1.0;
                ispike[i] = 0.0;
            }
            epoch[i] = reset_epoch;
        }
    };
    std::priority_queue<Ev, std::vector<Ev>, Later> q;
    // NetStim::initialize_cpu (netstim.cpp:207-239): one invl per started instance, in order
    for (int i = 0; i < n; i++) {
        if (ns.start[i] >= 0.0 && ns.number[i] > 0) {
            on[i] = 1.0;
            double iv = interval_of(i);
            double inv = iv;
            if (noise[i] != 0) inv = (1.0 - noise[i]) * iv + noise[i] * iv * rng.negexp(draws++);
            double ev = ns.start[i] + inv - ns.interval[i] * (1.0 - noise[i]);
            if (ev < 0.0) ev = 0.0;
            q.push(Ev{ev, i, kInit});
        }
    }
    std::vector<Ev> batch;
    for (int r = -1; r < nstep; r++) {
        const double t = r < 0 ? 0.0 : tstart[r];
        const double tt = t + dt / 2;
        const int step = r < 0 ? 0 : r;
        for (;;) {
            batch.clear();
            while (!q.empty() && !(q.top().t > tt)) {
                batch.push_back(q.top());
                q.pop();
            }
            int sent = 0;
            for (const Ev& e : batch) {
                const int i = e.id;
                touch(i);
                if (e.flag == kInit && on[i] == 1.0) {
                    reset_epoch++;  // init_sequence over every instance
                    touch(i);
                    q.push(Ev{t + 0.0, i, kSelf});
                    sent++;
                }
                if (e.flag == kSelf && on[i] == 1.0) {
                    ispike[i] += 1.0;
                    out_id.push_back(i);
                    out_step.push_back(step);
                    // next_invl: M draws; the firing instance's is the one read
                    double ev = interval_of(i);
                    if (rank[i] >= 0) ev = (1.0 - noise[i]) * ev + noise[i] * ev * rng.negexp(draws + (uint64_t)rank[i]);
                    draws += (uint64_t)M;
                    if (ispike[i] >= ns.number[i]) on[i] = 0.0;
                    if (on[i] == 1.0) {
                        q.push(Ev{t + ev, i, kSelf});
                        sent++;
                    }
                }
            }
            if (!sent) break;
        }
    }
}

}  // namespace hx
