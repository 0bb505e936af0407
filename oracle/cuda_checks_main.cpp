// Entry point for the reference's own GPU test suite, compiled against this
// library.  TEST INFRASTRUCTURE ONLY (built into oracle/_ref/).
//
// ParCIS/MX-KMeans tests/cuda_checks.cu holds three check functions
// (check_gemm_and_quantization :35-88, check_assignment_and_bounds :90-140,
// check_clustering :142-168) written against include/kmeans.cuh.  Its main()
// (:170-186) skips unless the GPU is SM120, so the recipe compiles that file with
// main renamed and this main calls the three checks directly on the B200.
#include <exception>
#include <iostream>

void check_gemm_and_quantization();
void check_assignment_and_bounds();
void check_clustering();

int main() {
    try {
        check_gemm_and_quantization();
        std::cout << "check_gemm_and_quantization passed" << std::endl;
        check_assignment_and_bounds();
        std::cout << "check_assignment_and_bounds passed" << std::endl;
        check_clustering();
        std::cout << "check_clustering passed" << std::endl;
        std::cout << "CUDA checks passed" << std::endl;
    } catch (const std::exception& e) {
        std::cerr << e.what() << '\n';
        return 1;
    }
    return 0;
}
