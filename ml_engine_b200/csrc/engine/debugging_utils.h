// debugging_utils.h -- the names ML_Engine's Includes/debugging_utils.h gives
// the programs built on it: the hyper-parameter constants, CheckError,
// SafeCudaMalloc, the Timing helper and the host-side print helpers, with
// the same signatures, so a use case that includes this header (directly or
// through engine.h) compiles unchanged.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <iostream>
#include <string>
#include <vector>

using str = std::string;

// Includes/debugging_utils.h:10-14
static constexpr float XAVIER = 6.0f;
static constexpr bool ADAMW = true;
static constexpr float NORM = 1.0f;
static constexpr float LEARNING_RATE = 1e-4f;
static constexpr bool SHOULDNORM = false;

// Synchronises the device; on a pending CUDA error prints `reason` and the
// error and exits(1) (Engine/debug.cu:15-25).
void CheckError(const str& reason);

// cudaMalloc of `size` elements; prints and exits(1) on failure.
template <typename T>
void SafeCudaMalloc(const str name, T*& pointer, size_t size) {
    const cudaError_t err = cudaMalloc((void**)&pointer, size * sizeof(T));
    if (err != cudaSuccess) {
        size_t free_b = 0, total_b = 0;
        cudaMemGetInfo(&free_b, &total_b);
        std::cerr << "Failed to allocate " << name << " of size " << size << ": " << cudaGetErrorString(err)
                  << " (" << (free_b >> 20) << " of " << (total_b >> 20) << " MB free)\n";
        pointer = nullptr;
        std::exit(1);
    }
}

// Wall-clock timing of a named region: start(), end() prints the elapsed
// milliseconds.
class Timing {
   public:
    explicit Timing(const str reason);
    ~Timing();
    void start();
    void end();

   private:
    std::chrono::time_point<std::chrono::high_resolution_clock> beg_;
    str what_;
    bool running_ = false;
};

inline void printMem(const char* label) {
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    std::printf("[%s] GPU free: %.2f MB\n", label, free_b / 1e6);
}

// elems values of a device array from `start`
template <typename T>
void printHeadGPU(const str name, T* d_ptr, int start, int elems, int total) {
    std::vector<T> h((size_t)total);
    cudaMemcpy(h.data(), d_ptr, sizeof(T) * (size_t)total, cudaMemcpyDeviceToHost);
    std::cout << "Printing dimensions for pointer: " << name << "\n";
    for (int i = start; i < start + elems && i < total; ++i) std::cout << h[(size_t)i] << "\t";
    std::cout << "\n _______________________________ \n";
}

namespace mle {
template <typename T>
void print_corner(const str& title, const T* d_ptr, int ch, int rows, int cols, int total) {
    std::vector<T> h((size_t)total);
    cudaMemcpy(h.data(), d_ptr, sizeof(T) * (size_t)total, cudaMemcpyDeviceToHost);
    std::cout << title;
    for (int c = 0; c < std::min(3, ch); ++c) {
        std::cout << "Channel " << c << ":\n";
        for (int r = 0; r < std::min(5, rows); ++r) {
            for (int k = 0; k < std::min(5, cols); ++k) std::cout << h[(size_t)(c * rows * cols + r * cols + k)] << "\t";
            std::cout << "\n";
        }
        std::cout << "------------------------------\n";
    }
}
}  // namespace mle

// the top-left 3 x 5 x 5 corner of a [ch, rows, cols] device tensor
template <typename T>
void printHeadGPU(const str name, const T* X, const int ch, const int rows, const int cols, const int total) {
    mle::print_corner("Printing dimensions for node " + name + "->output \n", X, ch, rows, cols, total);
}

template <typename T>
void printHeadGrad(const str name, const T* X, const int ch, const int rows, const int cols, const int total) {
    mle::print_corner("Printing dimensions for node " + name + "->grad \n", X, ch, rows, cols, total);
}
