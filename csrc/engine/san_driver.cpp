// Sanitizer driver for the CPU expert engine and the cold store: built together with engine.cpp, kernels.cpp and
// store.cpp under ThreadSanitizer or AddressSanitizer + UndefinedBehaviorSanitizer (no GPU involved), it exercises
// the paths that share state across threads:
//   * two plans (different shapes) calling forward / forward_decode from two host threads at once -- they share the
//     process-wide worker pool, whose job hand-off is the concurrency-critical part;
//   * a third thread pinning and unpinning RAM slots of the first plan and reading its slot table meanwhile;
//   * a cold-backed plan (6 RAM slots for 8 experts, 3 of them empty at start) whose misses are read from a cold
//     store file through the store's reader threads, checked bit-exactly against a fully resident plan.
// Exit code 0 when every result matches its single-threaded value; sanitizer reports make the run fail through the
// sanitizer's own exit code. Reference parity: tests/engine_san.cpp:1-260 (the reference's driver of the same
// three situations).
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "xt_engine.h"

namespace {

struct Experts {
    int E, H, I;
    std::vector<uint8_t> w13, w2, s13, s2;
    std::vector<float> g13, g2;
};

Experts make(int E, int H, int I, uint32_t seed) {
    Experts x{E, H, I, {}, {}, {}, {}, {}, {}};
    std::mt19937 rng(seed);
    auto fill = [&](std::vector<uint8_t> &v, size_t n, int lo, int hi) {
        v.resize(n);
        std::uniform_int_distribution<int> d(lo, hi);
        for (auto &b : v) b = uint8_t(d(rng));
    };
    fill(x.w13, size_t(E) * 2 * I * H / 2, 0, 255);
    fill(x.w2, size_t(E) * H * I / 2, 0, 255);
    fill(x.s13, size_t(E) * 2 * I * H / 16, 0x20, 0x30);   // E4M3 scales around 2^-3
    fill(x.s2, size_t(E) * H * I / 16, 0x20, 0x30);
    x.g13.assign(size_t(E) * 2, 1.f);
    x.g2.assign(size_t(E), 1.f);
    return x;
}

void *plan_of(const Experts &x, int slots, const int32_t *resident) {
    return xt_engine_create(x.H, x.I, x.E, 0, slots, 4, 0.f, 0, x.w13.data(), x.w2.data(), x.s13.data(),
                            x.s2.data(), x.g13.data(), x.g2.data(), resident);
}

struct Call {
    int m, k;
    std::vector<uint16_t> x;
    std::vector<int32_t> ids;
    std::vector<float> w;
};

Call make_call(int m, int k, int H, int E, uint32_t seed) {
    Call c{m, k, {}, {}, {}};
    std::mt19937 rng(seed);
    std::normal_distribution<float> n(0.f, 1.f);
    c.x.resize(size_t(m) * H);
    for (auto &v : c.x) {
        float f = n(rng);
        uint32_t u;
        std::memcpy(&u, &f, 4);
        v = uint16_t(u >> 16);
    }
    std::uniform_int_distribution<int> e(0, E - 1);
    std::uniform_real_distribution<float> u(0.1f, 1.f);
    c.ids.resize(size_t(m) * k);
    c.w.resize(size_t(m) * k);
    for (int t = 0; t < m; ++t)
        for (int j = 0; j < k; ++j) {
            c.ids[t * k + j] = (e(rng) + j * 3) % E;
            c.w[t * k + j] = u(rng);
        }
    return c;
}

std::vector<float> run(void *plan, const Call &c, int H, bool decode) {
    std::vector<float> y(size_t(c.m) * H);
    const int rc = decode ? xt_engine_forward_decode(plan, c.m, c.k, c.x.data(), c.ids.data(), c.w.data(), y.data())
                          : xt_engine_forward(plan, c.m, c.k, c.x.data(), c.ids.data(), c.w.data(), y.data());
    if (rc < 0) {
        std::fprintf(stderr, "forward failed: %s\n", xt_engine_error());
        std::exit(3);
    }
    return y;
}

bool same(const std::vector<float> &a, const std::vector<float> &b) {
    return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * sizeof(float)) == 0;
}

}  // namespace

int main(int argc, char **argv) {
    const std::string dir = argc > 1 ? argv[1] : "/tmp";
    int failures = 0;
    // two plans of different shapes, single-threaded references first
    const Experts a = make(8, 256, 128, 1), b = make(6, 512, 256, 2);
    void *pa = plan_of(a, a.E, nullptr), *pb = plan_of(b, b.E, nullptr);
    if (!pa || !pb) {
        std::fprintf(stderr, "create failed: %s\n", xt_engine_error());
        return 2;
    }
    const Call ca = make_call(5, 3, a.H, a.E, 11), cb = make_call(2, 4, b.H, b.E, 12);
    const std::vector<float> ra = run(pa, ca, a.H, false), rb = run(pb, cb, b.H, true);
    std::atomic<bool> stop{false};
    std::atomic<int> bad{0};
    std::thread t1([&] {
        for (int i = 0; i < 40; ++i)
            if (!same(run(pa, ca, a.H, false), ra)) bad++;
    });
    std::thread t2([&] {
        for (int i = 0; i < 40; ++i)
            if (!same(run(pb, cb, b.H, true), rb)) bad++;
    });
    std::thread t3([&] {   // pin / unpin slots of plan a while it computes, and read its table
        std::vector<int32_t> table(a.E);
        while (!stop.load()) {
            for (int e = 0; e < a.E; ++e) {
                const int s = xt_engine_slot_pin(pa, e);
                if (s >= 0) xt_engine_slot_unpin(pa, s);
            }
            xt_engine_slot_table(pa, table.data());
        }
    });
    t1.join();
    t2.join();
    stop = true;
    t3.join();
    if (bad) {
        std::fprintf(stderr, "concurrent plans: %d mismatching results\n", bad.load());
        ++failures;
    }
    // cold-backed plan: fewer RAM slots than experts, the rest in a cold store file
    const std::string path = dir + "/xt_san_cold.bin";
    const char *paths[1] = {path.c_str()};
    void *store = xt_cold_open(paths, 1, 2, 1);
    if (!store) {
        std::fprintf(stderr, "cold open failed: %s\n", xt_cold_error());
        return 2;
    }
    // a cold record: gate, up, gate scales, up scales, down, down scales, each padded to 512 bytes
    const size_t gw = size_t(a.I) * a.H / 2, gs = size_t(a.I) * a.H / 16;
    const size_t dw = size_t(a.H) * a.I / 2, ds = size_t(a.H) * a.I / 16;
    auto pad = [](size_t b) { return (b + 511) / 512 * 512; };
    const size_t per = pad(gw) * 2 + pad(gs) * 2 + pad(dw) + pad(ds);
    std::vector<int32_t> files(a.E, 0);
    std::vector<long long> offs(a.E);
    for (int e = 0; e < a.E; ++e) {
        offs[e] = (long long)(per * e);
        const void *pieces[6] = {a.w13.data() + e * 2 * gw, a.w13.data() + e * 2 * gw + gw,
                                 a.s13.data() + e * 2 * gs, a.s13.data() + e * 2 * gs + gs,
                                 a.w2.data() + e * dw, a.s2.data() + e * ds};
        const size_t sizes[6] = {gw, gw, gs, gs, dw, ds};
        if (xt_cold_write(store, 0, offs[e], pieces, sizes, 6) != 0) {
            std::fprintf(stderr, "cold write failed: %s\n", xt_cold_error());
            return 2;
        }
    }
    // 6 RAM slots, experts 0-2 resident, 3 empty: a call over experts 0-5 loads 3-5 from the store (and evicts on the
    // next calls as the decayed use counts change)
    const int32_t resident[6] = {0, 1, 2, -1, -1, -1};
    void *pc = plan_of(a, 6, resident);
    const Call cc = make_call(4, 3, a.H, 6, 21);
    const std::vector<float> rc_ref = run(pa, cc, a.H, false);
    std::vector<float> scores(a.E, 1.f);
    if (!pc || xt_engine_cold_attach(pc, store, files.data(), offs.data(), scores.data(), 64.f) != 0) {
        std::fprintf(stderr, "cold plan failed: %s\n", xt_engine_error());
        return 2;
    }
    for (int i = 0; i < 6; ++i)
        if (!same(run(pc, cc, a.H, i & 1), rc_ref)) {
            std::fprintf(stderr, "cold plan: result %d differs from the resident plan\n", i);
            ++failures;
            break;
        }
    xt_engine_destroy(pc);
    xt_cold_close(store);
    std::remove(path.c_str());
    xt_engine_destroy(pa);
    xt_engine_destroy(pb);
    std::printf("engine sanitizer driver: %s\n", failures ? "FAILED" : "ok");
    return failures ? 1 : 0;
}
