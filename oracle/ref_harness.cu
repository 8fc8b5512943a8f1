// Exposes the reference's own host-side UMMA known answer (reference_d,
// umma_throughput/umma_1sm.cu:566-575) through a C symbol so the oracle's
// restatement can be pinned against it. The reference file is included
// where it lies (never copied); its main() is renamed out of the way.
// Test infrastructure only.
#define main reference_umma_1sm_main
#include "umma_1sm.cu"
#undef main

extern "C" double ref_umma_reference_d(int row, int col, int depth) { return reference_d(row, col, depth); }
