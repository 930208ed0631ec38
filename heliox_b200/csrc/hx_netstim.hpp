// hx_netstim.hpp -- host generator of NetStim spike trains (see hx_netstim.cpp).
#pragma once

#include <vector>

namespace hx {

struct NetStimTable {
    int n = 0;
    const double *interval = nullptr, *number = nullptr, *start = nullptr, *noise = nullptr;
    int rng_mode = 0;
};

// Spikes of every NetStim over finitialize + nstep steps: instance index and
// the step at whose start it fires (0 for the delivery at finitialize, whose
// time t = 0 equals the start of step 0).  tstart[k] is the time at the start
// of step k, accumulated in half steps like Simulate::fadvance_cpu.
void netstim_trains(const NetStimTable& ns, const std::vector<double>& tstart, double dt, int nstep,
                    std::vector<int>& out_id, std::vector<int>& out_step);

}  // namespace hx
