// Minimal command-line parser for the task-1 driver.  Accepts the reference driver's options
// (results/naive_cycle6/src/main.cpp:95-118: -m -n -k, -w/--n_warmup, -t/--n_test, -h/--help) with the
// same defaults, plus additive ones: --seed, --dist normal|uniform, --lo, --hi, --json <path>.
// Forms accepted: "-m 4096", "-m=4096", "--m 4096", "--n_warmup=10".
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <stdexcept>
#include <string>

namespace playground
{
class Cli
{
public:
    Cli(int argc, const char* argv[])
    {
        for (int i = 1; i < argc; ++i) {
            std::string a = argv[i];
            if (a.size() < 2 || a[0] != '-') throw std::invalid_argument("unexpected argument '" + a + "'");
            a = a.substr(a[1] == '-' ? 2 : 1);
            std::string val;
            const auto eq = a.find('=');
            if (eq != std::string::npos) {
                val = a.substr(eq + 1);
                a = a.substr(0, eq);
            } else if (a != "h" && a != "help") {
                if (i + 1 >= argc) throw std::invalid_argument("option '" + a + "' needs a value");
                val = argv[++i];
            }
            values_[canonical(a)] = val;
        }
    }

    bool has(const std::string& key) const { return values_.count(key) != 0; }

    std::uint32_t u32(const std::string& key, std::uint32_t def) const
    {
        auto it = values_.find(key);
        return it == values_.end() ? def : static_cast<std::uint32_t>(std::stoul(it->second));
    }
    std::int64_t i64(const std::string& key, std::int64_t def) const
    {
        auto it = values_.find(key);
        return it == values_.end() ? def : std::stoll(it->second);
    }
    double f64(const std::string& key, double def) const
    {
        auto it = values_.find(key);
        return it == values_.end() ? def : std::stod(it->second);
    }
    std::string str(const std::string& key, const std::string& def) const
    {
        auto it = values_.find(key);
        return it == values_.end() ? def : it->second;
    }

    static const char* usage()
    {
        return "Playground Task1: General Matrix Multiplication\n"
               "  -m arg               Num of rows of A and C (default: 4096)\n"
               "  -n arg               Num of columns of B and C (default: 4096)\n"
               "  -k arg               Num of columns of A and rows of B (default: 4096)\n"
               "  -w, --n_warmup arg   Num of warmup rounds (default: 10)\n"
               "  -t, --n_test arg     Num of test rounds (default: 100)\n"
               "  -h, --help           Print usage\n"
               "      --seed arg       Input seed (default: std::random_device)\n"
               "      --dist arg       normal (default) or uniform\n"
               "      --lo arg, --hi arg   uniform range (default -1, 1)\n"
               "      --json arg       also write the result as one JSON line to this file\n"
               "      --gpus arg       split the rows over GPUs 0..arg-1 (vk_gemm_sharded; GPU versions)\n"
               "      --allgather arg  none | nccl (default) | pipelined | fused | nvls: all-gather of C\n";
    }

private:
    static std::string canonical(const std::string& k)
    {
        if (k == "w" || k == "n_warmup") return "w";
        if (k == "t" || k == "n_test") return "t";
        if (k == "h" || k == "help") return "h";
        return k;
    }
    std::map<std::string, std::string> values_;
};
}  // namespace playground
