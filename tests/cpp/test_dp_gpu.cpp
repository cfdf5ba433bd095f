// The fused ZeRO-1 step from C++ with no Python: one process per GPU, the
// library's data-parallel bootstrap (soar::optim::Communicator over
// soar_dp_init, soar::optim::ZeroOneAdamW over soar_dp_zero1_create).
//
//   test_dp_gpu <rank> <world> <id file> <output prefix> [device|nccl]
//
// Rank 0 writes NCCL's unique id to <id file>; the other ranks read it there.
// Every rank adds a second gradient buffer and the steps alternate between
// the two. Every rank steps 5 times on its own seeded bf16 gradient (loss scale 1024,
// growth every 2 clean steps, clip 1.0; +inf in rank 1's gradient at step 3,
// so that step is skipped everywhere) and writes its parameter buffer to
// <prefix>.rank<r>. Rank 0 also runs the same 5 steps as a single-GPU
// optimizer on the average of all ranks' gradients -- summed in fp32 in rank
// order, multiplied by 1/R once, rounded to bf16 once, the fused
// reduce-scatter's definition -- and checks: the step / skip / scale
// sequences equal; the parameters within 1 bf16 ulp of the single-GPU step
// (only the global norm's summation order differs); and every rank's
// parameter buffer identical to its own. Exit code 0 = pass.
#include <unistd.h>

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "soar_optim.hpp"

namespace {

constexpr uint64_t kN = 3000017;
constexpr uint64_t kBucket = 1000000;
constexpr int kSteps = 5;
constexpr int kInfStep = 3;

int g_failures = 0;
#define CHECK(cond, ...)                                      \
    do {                                                      \
        if (!(cond)) {                                        \
            std::printf("FAIL %s:%d: ", __FILE__, __LINE__);  \
            std::printf(__VA_ARGS__);                         \
            std::printf("\n");                                \
            ++g_failures;                                     \
        }                                                     \
    } while (0)

uint16_t to_bf16(float f) {  // round to nearest even (NaN never occurs here)
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
float from_bf16(uint16_t h) {
    const uint32_t u = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

std::vector<float> normals(uint64_t seed, size_t n, double std_dev) {
    std::vector<float> out(n);
    uint64_t s = seed;
    auto next = [&s]() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    for (size_t i = 0; i < n; i += 2) {
        const double u1 = (static_cast<double>(next() >> 11) + 1.0) * 0x1.0p-53;
        const double u2 = static_cast<double>(next() >> 11) * 0x1.0p-53;
        const double r = std::sqrt(-2.0 * std::log(u1)) * std_dev;
        out[i] = static_cast<float>(r * std::cos(2.0 * M_PI * u2));
        if (i + 1 < n) out[i + 1] = static_cast<float>(r * std::sin(2.0 * M_PI * u2));
    }
    return out;
}

// Rank r's bf16 gradient at step t under loss scale `scale`.
std::vector<uint16_t> grads_of(int r, int t, float scale) {
    const std::vector<float> g = normals(500 + 100 * static_cast<uint64_t>(r) + t, kN, 0.01);
    std::vector<uint16_t> out(kN);
    for (uint64_t i = 0; i < kN; ++i) out[i] = to_bf16(g[i] * scale);
    if (t == kInfStep && r == 1) out[123] = to_bf16(INFINITY);
    return out;
}

bool wait_for_file(const std::string& path, double seconds) {
    const auto end = std::chrono::steady_clock::now() + std::chrono::duration<double>(seconds);
    while (std::chrono::steady_clock::now() < end) {
        if (access(path.c_str(), R_OK) == 0) return true;
        std::this_thread::sleep_for(std::chrono::milliseconds(20));
    }
    return false;
}

int ordered(uint16_t h) {
    const int x = h;
    return (x & 0x8000) ? -(x & 0x7FFF) : x;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 5) {
        std::printf("usage: %s rank world id_file out_prefix [device|nccl]\n", argv[0]);
        return 2;
    }
    const int rank = std::atoi(argv[1]), world = std::atoi(argv[2]);
    const std::string id_file = argv[3], prefix = argv[4];
    const int sync = (argc > 5 && std::string(argv[5]) == "nccl") ? SOAR_DP_SYNC_NCCL
                                                                  : SOAR_DP_SYNC_DEVICE;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev < world) {
        std::printf("needs %d GPUs\n", world);
        return 77;
    }
    cudaSetDevice(rank);
    try {
        // the unique id, from rank 0 to the others through a file
        std::vector<unsigned char> id;
        if (rank == 0) {
            id = soar::optim::Communicator::unique_id();
            const std::string tmp = id_file + ".tmp";
            std::ofstream(tmp, std::ios::binary).write(reinterpret_cast<const char*>(id.data()),
                                                      static_cast<std::streamsize>(id.size()));
            std::rename(tmp.c_str(), id_file.c_str());
        } else {
            if (!wait_for_file(id_file, 60)) {
                std::printf("no unique id from rank 0\n");
                return 1;
            }
            id.resize(SOAR_DP_UNIQUE_ID_BYTES);
            std::ifstream(id_file, std::ios::binary)
                .read(reinterpret_cast<char*>(id.data()), static_cast<std::streamsize>(id.size()));
        }
        soar::optim::Communicator comm(rank, world, id, rank);

        std::vector<uint16_t> p0(kN);
        {
            const std::vector<float> p = normals(51, kN, 0.02);
            for (uint64_t i = 0; i < kN; ++i) p0[i] = to_bf16(p[i]);
        }
        soar::optim::AdamWOptions opts;
        opts.weight_decay = 0.01f;
        soar::optim::AdamWExtOptions ext;
        ext.layout = SOAR_LAYOUT_BF16_MIXED;
        ext.max_grad_norm = 1.0f;
        ext.use_loss_scaler = true;
        ext.init_scale = 1024.0f;
        ext.growth_interval = 2;
        ext.device = rank;
        soar::optim::ZeroOneAdamW z(comm, kN, kBucket, opts, ext, p0.data(), sync);
        // a second gradient buffer: the steps alternate between the two
        const int second = z.add_grads();
        CHECK(second == 1 && z.grads(0) != z.grads(1), "second gradient buffer (index %d)",
              second);

        // rank 0's single-GPU optimizer on the rank-averaged gradient
        uint16_t *ref_p = nullptr, *ref_g = nullptr;
        std::unique_ptr<soar::optim::AdamW> ref;
        if (rank == 0) {
            cudaMalloc(&ref_p, kN * 2);
            cudaMalloc(&ref_g, kN * 2);
            cudaMemcpy(ref_p, p0.data(), kN * 2, cudaMemcpyHostToDevice);
            std::vector<soar_tensor_desc> d;
            for (uint64_t s = 0; s < kN; s += kBucket)
                d.push_back({ref_p + s, ref_g + s, std::min(kBucket, kN - s), 0.01f});
            ref = std::make_unique<soar::optim::AdamW>(d, opts, ext);
        }
        float scale = ext.init_scale, ref_scale = ext.init_scale;
        std::vector<soar_step_info> mine, theirs;
        const float inv_r = 1.0f / static_cast<float>(world);
        for (int t = 1; t <= kSteps; ++t) {
            const std::vector<uint16_t> g = grads_of(rank, t, scale);
            z.use_grads((t - 1) % 2);
            cudaMemcpy(z.grads(), g.data(), kN * 2, cudaMemcpyHostToDevice);
            z.step();
            mine.push_back(z.info());
            scale = mine.back().loss_scale;
            if (ref) {
                std::vector<float> sum(kN, 0.0f);
                for (int q = 0; q < world; ++q) {
                    const std::vector<uint16_t> gq = grads_of(q, t, ref_scale);
                    for (uint64_t i = 0; i < kN; ++i) sum[i] += from_bf16(gq[i]);
                }
                std::vector<uint16_t> avg(kN);
                for (uint64_t i = 0; i < kN; ++i) avg[i] = to_bf16(sum[i] * inv_r);
                cudaMemcpy(ref_g, avg.data(), kN * 2, cudaMemcpyHostToDevice);
                ref->step();
                theirs.push_back(ref->info());
                ref_scale = theirs.back().loss_scale;
            }
        }
        cudaDeviceSynchronize();
        CHECK(z.error() == 0, "a device-side wait timed out");
        std::vector<uint16_t> out(kN);
        cudaMemcpy(out.data(), z.params(), kN * 2, cudaMemcpyDeviceToHost);
        {
            const std::string path = prefix + ".rank" + std::to_string(rank);
            std::ofstream(path + ".tmp", std::ios::binary)
                .write(reinterpret_cast<const char*>(out.data()), kN * 2);
            std::rename((path + ".tmp").c_str(), path.c_str());
        }
        CHECK(mine.back().step == kSteps - 1 && mine.back().skipped == 1,
              "step %llu skipped %llu", (unsigned long long)mine.back().step,
              (unsigned long long)mine.back().skipped);
        if (rank == 0) {
            for (int t = 0; t < kSteps; ++t)
                CHECK(mine[t].step == theirs[t].step && mine[t].skipped == theirs[t].skipped &&
                          mine[t].loss_scale == theirs[t].loss_scale,
                      "step %d: (%llu, %llu, %g) vs single GPU (%llu, %llu, %g)", t + 1,
                      (unsigned long long)mine[t].step, (unsigned long long)mine[t].skipped,
                      mine[t].loss_scale, (unsigned long long)theirs[t].step,
                      (unsigned long long)theirs[t].skipped, theirs[t].loss_scale);
            std::vector<uint16_t> rp(kN);
            cudaMemcpy(rp.data(), ref_p, kN * 2, cudaMemcpyDeviceToHost);
            int worst = 0;
            uint64_t off = 0;
            for (uint64_t i = 0; i < kN; ++i) {
                const int d = std::abs(ordered(out[i]) - ordered(rp[i]));
                worst = std::max(worst, d);
                off += d != 0;
            }
            CHECK(worst <= 1, "params differ from the single-GPU step by %d bf16 ulp", worst);
            for (int q = 1; q < world; ++q) {
                const std::string path = prefix + ".rank" + std::to_string(q);
                if (!wait_for_file(path, 120)) {
                    CHECK(false, "no parameters from rank %d", q);
                    continue;
                }
                std::vector<uint16_t> other(kN);
                std::ifstream(path, std::ios::binary)
                    .read(reinterpret_cast<char*>(other.data()), kN * 2);
                CHECK(std::memcmp(other.data(), out.data(), kN * 2) == 0,
                      "rank %d's parameters differ from rank 0's", q);
            }
            std::printf("rank 0: max %d bf16 ulp from the single-GPU step (%llu elements off)\n",
                        worst, (unsigned long long)off);
            cudaFree(ref_p);
            cudaFree(ref_g);
        }
    } catch (const std::exception& ex) {
        std::printf("rank %d: %s\n", rank, ex.what());
        return 1;
    }
    if (g_failures) {
        std::printf("rank %d: %d FAILURE(S)\n", rank, g_failures);
        return 1;
    }
    std::printf("rank %d: DP C++ TEST PASSED\n", rank);
    return 0;
}
