// ref_harness.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Runs the reference's own CPU integrator on a CoreNEURON-format model
// directory (plus halfgap.i32, HalfGap (instance, source node) pairs replayed
// through Simulate::add_gap_source/add_gap_target) and writes the voltage
// trace at the requested nodes:
//   hxref_run <dir> <permute_type> <dt> <nstep> <v_init> <probes.i32> <trace.f64> <spike_dir>
// It follows the reference's own driver (src/main.cpp:180-233): read_coredat,
// Simulate(CPU), data_format_trans, finitialize, then fadvance per step (the
// trace is read from the group's voltage vector after every step, like
// LearnRuntime::simulate_output_vs_into), and output_spikes into spike_dir.
// permute_type 0 (the reference's CPU default, src/main.cpp:149-152) keeps
// node i of the files at group node i; types 1 and 3 (the reference's
// default in python_lib/heliox_learn/runtime.py:13) let read_coredat permute
// the nodes (src/io/read_coredat.cpp:825-875, permute_order.cpp:145-210) and
// solve with cpu_solve_permute1 / cpu_solve_permute3 (src/simulate.cpp:
// 583-713); probes are then read at the permuted index (the group's
// permute[i] is where file node i went).  HalfGap wiring is supported for
// type 0 only.  The wall time of finitialize plus the fadvance loop (the
// reference's integration alone, without loading or output) is printed as
// "HXREF_FADVANCE_S <seconds>".
//
//   hxref_run_gpu <same arguments> gpu|gpu-time
// (the binary linked against the real CUDA runtime, oracle/_ref/hxref_run_gpu)
// runs the reference's GPU integrator instead (Simulate(GPU): fadvance_gpu,
// src/simulate.cu:722-771, its mechanism kernels and cuda_solve_matrix):
// "gpu" copies the voltages back after every step to record the probes;
// "gpu-time" records only the initial and final states and times the fadvance
// loop between two device synchronisations (HXREF_FADVANCE_S).
//
//   hxref_run --adam <n> <steps> <lr> <inv_record_steps> <beta1> <beta2> <eps> <impedance> <in.f64> <out.f64>
// runs the reference's AdamOptimizer (src/optimizer/optimizer.cpp) on the CPU:
// in.f64 holds n initial weights followed by steps x n gradients; out.f64
// receives the weights after every step (steps x n) and the final m and v.
#include <cuda_runtime_api.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "coredat_to_innerdat.h"
#include "read_coredat.h"
#include "optimizer/optimizer.h"
#include "simulate.h"

extern int permute_type;

static int run_adam(int argc, char** argv) {
    if (argc != 12) return 2;
    const int n = std::atoi(argv[2]), steps = std::atoi(argv[3]);
    const double lr = std::atof(argv[4]), inv = std::atof(argv[5]);
    OptimizerHyperParams hp;
    hp.beta1 = std::atof(argv[6]);
    hp.beta2 = std::atof(argv[7]);
    hp.epsilon = std::atof(argv[8]);
    const double imp = std::atof(argv[9]);
    std::vector<double> in((size_t)n * (steps + 1));
    FILE* f = std::fopen(argv[10], "rb");
    if (!f || std::fread(in.data(), sizeof(double), in.size(), f) != in.size()) return 3;
    std::fclose(f);
    std::vector<double> w(in.begin(), in.begin() + n), g(n, 0.0);
    AdamOptimizer opt(CPU);
    opt.configure(hp);
    for (int i = 0; i < n; i++) {
        OptimizerParam prm;
        prm.weight_cpu = {&w[i]};
        prm.grad_cpu = {&g[i]};
        prm.impedance = imp;
        if (opt.add_param(prm) < 0) return 4;
    }
    std::vector<double> out;
    for (int s = 0; s < steps; s++) {
        for (int i = 0; i < n; i++) g[i] = in[(size_t)(s + 1) * n + i];
        opt.step(lr, inv);
        out.insert(out.end(), w.begin(), w.end());
    }
    long long sc = 0;
    std::vector<double> m, v;
    opt.export_state(sc, m, v);
    out.insert(out.end(), m.begin(), m.end());
    out.insert(out.end(), v.begin(), v.end());
    f = std::fopen(argv[11], "wb");
    if (!f) return 3;
    std::fwrite(out.data(), sizeof(double), out.size(), f);
    std::fclose(f);
    return 0;
}

int main(int argc, char** argv) {
    if (argc > 1 && std::string(argv[1]) == "--adam") return run_adam(argc, argv);
    if (argc != 9 && argc != 10) {
        std::fprintf(stderr, "usage: %s dir permute_type dt nstep v_init probes.i32 trace.f64 spike_dir [gpu|gpu-time]\n",
                     argv[0]);
        return 2;
    }
    const std::string gmode = argc == 10 ? argv[9] : "";
    if (!gmode.empty() && gmode != "gpu" && gmode != "gpu-time") {
        std::fprintf(stderr, "mode must be gpu or gpu-time\n");
        return 2;
    }
    const Mode mode = gmode.empty() ? CPU : GPU;
    const bool every_step = gmode != "gpu-time";
    const std::string dir = argv[1];
    const int ptype = std::atoi(argv[2]);
    const double dt = std::atof(argv[3]);
    const int nstep = std::atoi(argv[4]);
    const double v_init = std::atof(argv[5]);
    if (ptype != 0 && ptype != 1 && ptype != 3) {
        std::fprintf(stderr, "permute type must be 0, 1 or 3\n");
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
    Simulate* sim = new Simulate(mode, BufferEnable::NONE);
    sim->dt = dt;
    sim->tstop = nstep * dt;
    sim->output_folder = argv[8];
    data_format_trans(sim->neuron_group_list, arr, ngroup, mode, sim->dt);
    for (int i = 0; i < ngroup; i++) delete arr[i];
    sim->permute_type = ptype;
    // HalfGap vgap and gapjunction_noptr vpre of instance i follow the voltage
    // of a source node, wired through the reference's gap API (pairs written
    // by the exporter)
    for (const auto& [fname, mech, var] : {std::tuple<const char*, const char*, const char*>{"halfgap.i32", "HalfGap", "vgap"},
                                           {"gapnoptr.i32", "gapjunction_noptr", "vpre"}}) {
        FILE* f = std::fopen((dir + "/" + fname).c_str(), "rb");
        if (f && ptype != 0) {
            std::fprintf(stderr, "%s wiring needs permute type 0\n", mech);
            return 2;
        }
        if (f) {
            int pr[2];
            while (std::fread(pr, sizeof(int), 2, f) == 2) {
                const int sid = sim->add_gap_source("global", "v", pr[1]);
                if (sid < 0 || sim->add_gap_target(sid, mech, var, pr[0]) != 0) {
                    std::fprintf(stderr, "%s wiring failed for instance %d\n", mech, pr[0]);
                    return 4;
                }
            }
            std::fclose(f);
        }
    }
    std::vector<VarDescriptor> monitors;
    sim->init_monitor_data_sets(monitors);
    const auto t0 = std::chrono::steady_clock::now();
    sim->finitialize(v_init);
    HelioXroupData* g = sim->neuron_group_list[0];
    if (g->permute)
        for (int& q : probes) q = g->permute[q];
    std::vector<double> trace((size_t)(nstep + 1) * probes.size());
    auto record = [&](int row) {
        if (mode == GPU) g->vecdata_v->update_cpu_data_from_gpu();
        const double* v = g->vecdata_v->get_cpu_data();
        for (size_t q = 0; q < probes.size(); q++) trace[(size_t)row * probes.size() + q] = v[probes[q]];
    };
    record(0);
    auto t1 = t0;
    if (mode == GPU && !every_step) {
        cudaDeviceSynchronize();
        t1 = std::chrono::steady_clock::now();  // gpu-time: the fadvance loop alone
    }
    for (int k = 0; k < nstep; k++) {
        sim->fadvance();
        if (every_step) record(k + 1);
    }
    if (mode == GPU) cudaDeviceSynchronize();
    const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t1).count();
    if (!every_step) record(nstep);
    if (mode == GPU) {
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            std::fprintf(stderr, "CUDA error: %s\n", cudaGetErrorString(e));
            return 5;
        }
    }
    std::printf("HXREF_FADVANCE_S %.9f\n", secs);
    std::fflush(stdout);
    sim->output_spikes();
    FILE* f = std::fopen(argv[7], "wb");
    if (!f) return 3;
    std::fwrite(trace.data(), sizeof(double), trace.size(), f);
    std::fclose(f);
    return 0;
}
