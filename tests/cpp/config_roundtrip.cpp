// ConfigManager save -> defaults -> load round trip (tests/test_config_roundtrip.py, no GPU):
// every value save_to_file writes must come back exactly, floats included. Prints "ok" or the
// fields that differ.
//
//   config_roundtrip <scratch file>
#include <cstdio>
#include <string>

#include "vk_symbiote/ConfigManager.h"

using namespace vk_symbiote;

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    ConfigManager& cm = ConfigManager::instance();
    MemoryConfig m;
    m.vram_budget_gb = 48.125f;
    m.ram_budget_gb = 12.3456f;
    m.prefetch_lookahead = 5;
    m.eviction_aggression = 0.725f;
    m.enable_compression = false;
    cm.set_memory(m);
    PerformanceConfig p;
    p.enable_gpu = false;
    p.enable_profiling = true;
    p.use_fp16_math = false;
    cm.set_performance(p);
    BenchmarkConfig b;
    b.warmup_tokens = 7;
    b.benchmark_tokens = 123;
    b.iterations = 4;
    cm.set_benchmark(b);
    ParallelConfig par;
    par.tp_size = 4;
    par.device = 3;
    cm.set_parallel(par);
    cm.set_model_path("/models/llama 7b.gguf");
    if (!cm.save_to_file(argv[1])) return 3;
    cm.set_defaults();
    cm.load_from_file(argv[1]);
    std::string bad;
    auto chk = [&](bool ok, const char* what) {
        if (!ok) bad += std::string(" ") + what;
    };
    chk(cm.memory().vram_budget_gb == 48.125f, "vram_budget_gb");
    chk(cm.memory().ram_budget_gb == 12.3456f, "ram_budget_gb");
    chk(cm.memory().prefetch_lookahead == 5, "prefetch_lookahead");
    chk(cm.memory().eviction_aggression == 0.725f, "eviction_aggression");
    chk(!cm.memory().enable_compression, "enable_compression");
    chk(!cm.performance().enable_gpu && cm.performance().enable_profiling && !cm.performance().use_fp16_math,
        "performance flags");
    chk(cm.benchmark().warmup_tokens == 7 && cm.benchmark().benchmark_tokens == 123 && cm.benchmark().iterations == 4,
        "benchmark");
    chk(cm.parallel().tp_size == 4 && cm.parallel().device == 3, "parallel");
    chk(cm.model_path() == "/models/llama 7b.gguf", "model path");
    printf("%s\n", bad.empty() ? "ok" : ("differ:" + bad).c_str());
    return 0;
}
