// ref_harness.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Runs the reference's own CPU integrator on a CoreNEURON-format model
// directory and writes the voltage trace at the requested nodes:
//   hxref_run <dir> <permute_type> <dt> <nstep> <v_init> <probes.i32> <trace.f64> <spike_dir>
// It follows the reference's own driver (src/main.cpp:180-233): read_coredat,
// Simulate(CPU), data_format_trans, finitialize, then fadvance per step (the
// trace is read from the group's voltage vector after every step, like
// LearnRuntime::simulate_output_vs_into), and output_spikes into spike_dir.
// Only permute type 0 (the reference's CPU default, src/main.cpp:149-152) is
// used, so reference node i is the group's node i.
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <string>
#include <vector>

#include "coredat_to_innerdat.h"
#include "read_coredat.h"
#include "simulate.h"

extern int permute_type;

int main(int argc, char** argv) {
    if (argc != 9) {
        std::fprintf(stderr, "usage: %s dir permute_type dt nstep v_init probes.i32 trace.f64 spike_dir\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1];
    const int ptype = std::atoi(argv[2]);
    const double dt = std::atof(argv[3]);
    const int nstep = std::atoi(argv[4]);
    const double v_init = std::atof(argv[5]);
    if (ptype != 0) {
        std::fprintf(stderr, "only permute type 0 is supported by this harness\n");
        return 2;
    }
    std::vector<int> probes;
    {
        FILE* f = std::fopen(argv[6], "rb");
        if (!f) return 3;
        int x;
        while (std::fread(&x, sizeof(int), 1, f) == 1) probes.push_back(x);
        std::fclose(f);
    }
    permute_type = ptype;
    std::unique_ptr<coreneuron::CoreData*[]> arr;
    const std::string files = dir + "/files.dat";
    int ngroup = read_coredat(arr, dir.c_str(), files.c_str(), 0, false, 1000);
    Simulate* sim = new Simulate(CPU, BufferEnable::NONE);
    sim->dt = dt;
    sim->tstop = nstep * dt;
    sim->output_folder = argv[8];
    data_format_trans(sim->neuron_group_list, arr, ngroup, CPU, sim->dt);
    for (int i = 0; i < ngroup; i++) delete arr[i];
    sim->permute_type = ptype;
    std::vector<VarDescriptor> monitors;
    sim->init_monitor_data_sets(monitors);
    sim->finitialize(v_init);
    HelioXroupData* g = sim->neuron_group_list[0];
    std::vector<double> trace((size_t)(nstep + 1) * probes.size());
    auto record = [&](int row) {
        const double* v = g->vecdata_v->get_cpu_data();
        for (size_t q = 0; q < probes.size(); q++) trace[(size_t)row * probes.size() + q] = v[probes[q]];
    };
    record(0);
    for (int k = 0; k < nstep; k++) {
        sim->fadvance();
        record(k + 1);
    }
    sim->output_spikes();
    FILE* f = std::fopen(argv[7], "wb");
    if (!f) return 3;
    std::fwrite(trace.data(), sizeof(double), trace.size(), f);
    std::fclose(f);
    return 0;
}
