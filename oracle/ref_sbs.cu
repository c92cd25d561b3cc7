// ref_sbs.cu -- build harness for the reference's step-by-step (time-driven)
// CUDA programs, the reported baseline the spec names beside vdttfs_cuda:
// task1_lenet_mnist/stepbystep_cuda/snn_mnist_stepbystep.cu,
// task2_vgg16_cifar10/stepbystep_cuda/bench_vgg_timedriven_baseline.cu and
// task2_vgg16_cifar10/stepbystep_lut_cuda/bench_vgg_timedriven_lut.cu.
//
// TEST INFRASTRUCTURE ONLY (output: oracle/_ref/libref_sbs_*.so, git-ignored).
// The program is #included unmodified from REF_SRC at build time; its `main`
// is renamed and run as is by ref_sbs_run inside a directory that holds the
// files it opens by relative path (exported_models/..., dataset_downloaded/...),
// so the timing and the throughput it prints are the program's own.
#define main ref_sbs_program_main
#include REF_SRC
#undef main

#include <unistd.h>

#include <climits>
#include <cstdio>

extern "C" int ref_sbs_run(const char* workdir) {
    char old[PATH_MAX];
    if (!getcwd(old, sizeof(old))) return -1;
    if (chdir(workdir) != 0) return -2;
    const int rc = ref_sbs_program_main();
    fflush(stdout);
    std::cout.flush();
    if (chdir(old) != 0) return -3;
    return rc;
}
