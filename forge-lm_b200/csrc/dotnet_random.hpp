// dotnet_random.hpp — the uniform stream of `new System.Random(seed)`.
//
// The reference draws one (float)rng.NextDouble() per sampled token
// (src/LLM.Core/Inference/Sampler.cs:61) from `new Random(seed)`
// (src/LLM.Cli/Program.cs:664, 730).  .NET seeds that generator with the
// published subtractive method of Knuth (TAOCP vol. 2, 3.2.2) in its "compat"
// variant: a 55-entry lagged table (lags 21/55) and NextDouble() =
// sample * (1.0 / int.MaxValue).  No .NET runtime exists on this build host,
// so agreement with a real .NET stream is not pinned by a test here.
#pragma once
#include <cstdint>
#include <cstring>

namespace fb2 {

class DotNetRandom {
    // C# int arithmetic wraps (unchecked context); so does this.
    static int32_t wsub(int32_t a, int32_t b) { return (int32_t)((uint32_t)a - (uint32_t)b); }
    static int32_t wadd(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }

public:
    explicit DotNetRandom(int32_t seed = 0) { reseed(seed); }

    void reseed(int32_t seed) {
        constexpr int32_t kBig = 2147483647, kSeed = 161803398;
        std::memset(t_, 0, sizeof(t_));
        int32_t sub = (seed == INT32_MIN) ? kBig : (seed < 0 ? -seed : seed);
        int32_t mj = kSeed - sub;
        t_[55] = mj;
        int32_t mk = 1, ii = 0;
        for (int i = 1; i < 55; i++) {
            ii += 21;
            if (ii >= 55) ii -= 55;
            t_[ii] = mk;
            mk = wsub(mj, mk);
            if (mk < 0) mk = wadd(mk, kBig);
            mj = t_[ii];
        }
        for (int k = 1; k < 5; k++)
            for (int i = 1; i < 56; i++) {
                int n = i + 30;
                if (n >= 55) n -= 55;
                t_[i] = wsub(t_[i], t_[1 + n]);
                if (t_[i] < 0) t_[i] = wadd(t_[i], kBig);
            }
        a_ = 0;
        b_ = 21;
    }

    int32_t next_sample() {
        constexpr int32_t kBig = 2147483647;
        int32_t a = a_ + 1;
        if (a >= 56) a = 1;
        int32_t b = b_ + 1;
        if (b >= 56) b = 1;
        int32_t v = wsub(t_[a], t_[b]);
        if (v == kBig) v--;
        if (v < 0) v = wadd(v, kBig);
        t_[a] = v;
        a_ = a;
        b_ = b;
        return v;
    }

    double next_double() { return next_sample() * (1.0 / 2147483647.0); }

private:
    int32_t t_[56];
    int32_t a_ = 0, b_ = 21;
};

}  // namespace fb2
