// Exercises the C++ host mirror (include/g4sampler.hpp) over the C ABI.
//   host_mirror cpu
//       defaults and error reporting; expects no usable GPU
//   host_mirror gpu <logits.f32 file> <V> <u> <T> <K> <P> <cap>
//       prints the token TSampler::DoSample returns for that row
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "g4sampler.hpp"

static int cpu_mode()
{
    g4::TSamplingParams p;
    if (p.temperature != 1.0f || p.top_k != 64 || p.top_p != 0.95f || p.repetition_penalty != 1.0f) {
        std::puts("bad defaults");
        return 1;
    }
    g4::TSampler s;
    std::vector<float> row(100, 0.0f);
    if (s.DoSample(p, row.data(), 0.5) != -1 || s.GetErrors().empty()) {
        std::puts("DoSample before Init must fail with an error");
        return 1;
    }
    if (s.Init(0, 4, 1000, 30.0f)) {
        std::puts("Init unexpectedly succeeded");
        return 1;
    }
    std::printf("%s\n", s.GetErrors().back().c_str());
    return 0;
}

static int gpu_mode(int argc, char **argv)
{
    if (argc < 9) return 2;
    const int V = std::atoi(argv[3]);
    std::vector<float> row(V);
    FILE *f = std::fopen(argv[2], "rb");
    if (!f || std::fread(row.data(), sizeof(float), V, f) != (size_t)V) return 3;
    std::fclose(f);
    g4::TSamplingParams p;
    p.temperature = (float)std::atof(argv[5]);
    p.top_k = std::atoi(argv[6]);
    p.top_p = (float)std::atof(argv[7]);
    g4::TSampler s;
    if (!s.Init(0, 1, V, (float)std::atof(argv[8]))) {
        std::printf("init failed: %s\n", s.GetErrors().back().c_str());
        return 4;
    }
    const int tok = s.DoSample(p, row.data(), std::atof(argv[4]));
    if (tok < 0 && !s.GetErrors().empty()) std::printf("error: %s\n", s.GetErrors().back().c_str());
    std::printf("token %d\n", tok);
    return 0;
}

int main(int argc, char **argv)
{
    if (argc >= 2 && !std::strcmp(argv[1], "cpu")) return cpu_mode();
    if (argc >= 2 && !std::strcmp(argv[1], "gpu")) return gpu_mode(argc, argv);
    return 2;
}
