// CPU expert engine (see xt_engine.h for the contract).
//
// Structure:
//  * Topology: NUMA nodes with allowed CPUs, from sysfs and sched_getaffinity (one node when sysfs says nothing).
//  * Pool: one process-wide set of worker threads, each pinned to a CPU of one node. Workers spin for XTIER_SPIN_US on
//    a generation word, then sleep on it with futex; the caller bumps the generation to start a job and joins the work.
//  * Plan: per node, a shard of every expert slot: rows [n*I/N, (n+1)*I/N) of gate and up, rows [n*H/N, ...) of down,
//    with their block scales, each piece 4 KiB aligned (so cold reads land with O_DIRECT). Shards are mbind()-ed to
//    their node and advised to use huge pages.
//  * forward: routes are grouped per expert (ascending id) into micro-groups of <= 8 tokens. Phase 1 tasks compute
//    row blocks of SwiGLU(gate x, up x) per group on the shard's node; phase 2 tasks own blocks of output rows and sum
//    every group's weighted down projection into them in group order, so no two tasks write one element and the
//    result does not depend on the thread count.
// Reference parity: csrc/engine/engine.cpp (worker pool :391-534, NUMA shards :360-386, phases :956-1058, micro-groups
// :1257-1300, tail skip :1227-1254, RAM slots and cold reads :1191-1225 / :1325-1440). The design here is its own: one
// library with per-function ISA targets instead of per-ISA builds behind a dlopen shim, one generic kernel per ISA.
#include "../include/xt_engine.h"
#include "kernels.h"

#include <errno.h>
#include <linux/futex.h>
#include <pthread.h>
#include <sched.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <ctype.h>
#include <math.h>

#include <algorithm>
#include <atomic>
#include <stdexcept>
#include <chrono>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace xt {

static thread_local std::string g_error;
static void set_error(const std::string &s) { g_error = s; }

static double now_us() {
    return std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

static int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

// ------------------------------------------------------------------------------------------------ topology
static std::vector<int> parse_cpulist(const std::string &s) {
    std::vector<int> out;
    size_t i = 0;
    while (i < s.size()) {
        while (i < s.size() && (s[i] == ',' || s[i] == ' ' || s[i] == '\n')) ++i;
        if (i >= s.size()) break;
        int a = 0, b;
        while (i < s.size() && isdigit(s[i])) a = a * 10 + (s[i++] - '0');
        b = a;
        if (i < s.size() && s[i] == '-') {
            ++i;
            b = 0;
            while (i < s.size() && isdigit(s[i])) b = b * 10 + (s[i++] - '0');
        }
        for (int c = a; c <= b; ++c) out.push_back(c);
    }
    return out;
}

static std::string read_file(const std::string &path) {
    FILE *f = fopen(path.c_str(), "r");
    if (!f) return "";
    char buf[4096];
    size_t n = fread(buf, 1, sizeof buf - 1, f);
    fclose(f);
    buf[n] = 0;
    return buf;
}

struct Topology {
    std::vector<std::vector<int>> node_cpus;   // allowed CPUs per node that has any
    std::vector<int> node_ids;
};

static Topology read_topology() {
    Topology t;
    cpu_set_t allowed;
    CPU_ZERO(&allowed);
    const char *wc = getenv("XTIER_WORKER_CPUS");   // a placement's worker CPUs (else the process's affinity)
    if (wc && *wc) {
        for (int c : parse_cpulist(wc))
            if (c >= 0 && c < CPU_SETSIZE) CPU_SET(c, &allowed);
    }
    if (CPU_COUNT(&allowed) == 0) sched_getaffinity(0, sizeof allowed, &allowed);
    for (int n = 0; n < 64; ++n) {
        std::string s = read_file("/sys/devices/system/node/node" + std::to_string(n) + "/cpulist");
        if (s.empty()) continue;
        std::vector<int> cpus;
        for (int c : parse_cpulist(s))
            if (c < CPU_SETSIZE && CPU_ISSET(c, &allowed)) cpus.push_back(c);
        if (!cpus.empty()) {
            t.node_cpus.push_back(cpus);
            t.node_ids.push_back(n);
        }
    }
    if (t.node_cpus.empty()) {
        std::vector<int> cpus;
        for (int c = 0; c < CPU_SETSIZE; ++c)
            if (CPU_ISSET(c, &allowed)) cpus.push_back(c);
        t.node_cpus.push_back(cpus);
        t.node_ids.push_back(0);
    }
    return t;
}

// Worker CPUs for `threads` workers: spread evenly over the nodes, each node's share from its allowed CPUs
static std::vector<std::vector<int>> worker_cpus(const Topology &t, int threads) {
    int N = int(t.node_cpus.size());
    std::vector<std::vector<int>> out(N);
    for (int i = 0; i < threads; ++i) {
        int n = i % N, j = i / N;
        const auto &c = t.node_cpus[n];
        out[n].push_back(c.empty() ? -1 : c[j % c.size()]);
    }
    return out;
}

// ------------------------------------------------------------------------------------------------ worker pool
static long futex(std::atomic<uint32_t> *addr, int op, uint32_t val) {
    return syscall(SYS_futex, reinterpret_cast<uint32_t *>(addr), op, val, nullptr, nullptr, 0);
}

struct Job {
    virtual void run(int worker, int node) = 0;
    virtual ~Job() {}
};

class Pool {
  public:
    int nthreads = 0, nnodes = 1;
    std::vector<int> worker_node;
    std::mutex use;   // one job at a time (plans share the pool)

    Pool(const Topology &topo, int threads) {
        nnodes = int(topo.node_cpus.size());
        if (threads < nnodes) threads = nnodes;
        threads -= threads % nnodes;
        nthreads = threads;
        spin_us = env_int("XTIER_SPIN_US", 200);
        auto cpus = worker_cpus(topo, threads);
        for (int n = 0; n < nnodes; ++n)
            for (size_t j = 0; j < cpus[n].size(); ++j) {
                worker_node.push_back(n);
                worker_cpu.push_back(cpus[n][j]);
            }
        for (int i = 0; i < nthreads; ++i) threads_.emplace_back([this, i] { loop(i); });
    }

    ~Pool() {
        stop.store(true);
        gen.fetch_add(1);
        futex(&gen, FUTEX_WAKE_PRIVATE, 0x7fffffff);
        for (auto &t : threads_) t.join();
    }

    // Runs job on every worker; the caller waits (spinning) until all returned.
    void run(Job *j) {
        job = j;
        done.store(0, std::memory_order_relaxed);
        gen.fetch_add(1, std::memory_order_release);
        if (sleepers.load(std::memory_order_acquire) > 0) futex(&gen, FUTEX_WAKE_PRIVATE, 0x7fffffff);
        while (done.load(std::memory_order_acquire) < nthreads) _mm_pause_();
        job = nullptr;
    }

    // Spinning barrier among the workers of the current job (generation-counted).
    void barrier() {
        uint32_t g = bar_gen.load(std::memory_order_acquire);
        if (bar_count.fetch_add(1, std::memory_order_acq_rel) + 1 == nthreads) {
            bar_count.store(0, std::memory_order_relaxed);
            bar_gen.fetch_add(1, std::memory_order_release);
        } else {
            while (bar_gen.load(std::memory_order_acquire) == g) _mm_pause_();
        }
    }

  private:
    std::vector<std::thread> threads_;
    std::vector<int> worker_cpu;
    std::atomic<uint32_t> gen{0};
    std::atomic<int> sleepers{0}, done{0};
    std::atomic<uint32_t> bar_gen{0};
    std::atomic<int> bar_count{0};
    std::atomic<bool> stop{false};
    Job *volatile job = nullptr;
    int spin_us = 200;

    static inline void _mm_pause_() { __builtin_ia32_pause(); }

    void loop(int i) {
        if (worker_cpu[i] >= 0) {
            cpu_set_t set;
            CPU_ZERO(&set);
            CPU_SET(worker_cpu[i], &set);
            pthread_setaffinity_np(pthread_self(), sizeof set, &set);
        }
        uint32_t seen = 0;   // the initial generation: a worker that starts late still sees the first job
        for (;;) {
            double t0 = now_us();
            uint32_t g;
            int spins = 0;
            while ((g = gen.load(std::memory_order_acquire)) == seen) {
                _mm_pause_();
                if (++spins == 256) {
                    spins = 0;
                    if (now_us() - t0 > spin_us) {
                        sleepers.fetch_add(1);
                        if (gen.load(std::memory_order_acquire) == seen) futex(&gen, FUTEX_WAIT_PRIVATE, seen);
                        sleepers.fetch_sub(1);
                        t0 = now_us();
                    }
                }
            }
            seen = g;
            if (stop.load()) return;
            Job *j = job;
            if (j) j->run(i, worker_node[i]);
            done.fetch_add(1, std::memory_order_acq_rel);
        }
    }
};

static std::mutex g_pool_mutex;
static Pool *g_pool = nullptr;
static Topology g_topo;

static Pool *get_pool(int threads) {
    std::lock_guard<std::mutex> lk(g_pool_mutex);
    if (!g_pool) {
        g_topo = read_topology();
        if (threads <= 0) {
            int all = 0;
            for (auto &c : g_topo.node_cpus) all += int(c.size());
            threads = std::max(1, all - 1);
        }
        g_pool = new Pool(g_topo, threads);
    }
    return g_pool;
}

static const Kernels *pick_kernels() {
    const char *isa = getenv("XTIER_ISA");
    std::string want = isa ? isa : "auto";
    if (want == "scalar") return kernels_scalar();
    if (want == "avx2") return kernels_avx2() ? kernels_avx2() : kernels_scalar();
    if (const Kernels *k = kernels_avx512()) return k;
    if (want == "avx512") return nullptr;
    if (const Kernels *k = kernels_avx2()) return k;
    return kernels_scalar();
}

// ------------------------------------------------------------------------------------------------ plan
static size_t pad4k(size_t b) { return (b + 4095) & ~size_t(4095); }

struct Shard {   // one node's part of every slot
    uint8_t *base = nullptr;
    size_t bytes = 0;
    size_t piece_off[6], piece_bytes[6], stride;   // per slot
    uint8_t *piece(int slot, int p) const { return base + size_t(slot) * stride + piece_off[p]; }
};

struct Group {   // one expert, <= MAX_TOK tokens
    int slot;    // index into the shard (routed slot or slots + shared index)
    int ntok;
    int tok[MAX_TOK];
    float w[MAX_TOK];
    float g_gate, g_up, g_down;
};

struct ColdStore;   // store.cpp

struct Plan {
    int H, I, E, shared, slots, fmt, nodes;
    float limit, alpha = 1.f, beta = 0.f;
    const Kernels *K;
    Pool *pool;
    std::vector<Shard> shards;
    std::vector<float> g13, g2;           // per slot (+shared): gate, up / down multipliers
    std::vector<float> eg13, eg2;         // per routed expert (optional): copied into a slot when the expert lands
    std::vector<int> slot_of, expert_of;  // expert -> slot, slot -> expert
    std::vector<int> pins;
    std::atomic<int> busy{0};
    // scratch
    std::vector<uint8_t> xprep, midprep;
    std::vector<Group> groups;
    double t_gate = 0, t_down = 0;
    // tail skip
    int tail_keep = 0, tail_total = 0, tail_tokens = 8;
    double tail_stats[3] = {0, 0, 0};
    // cold
    void *cold = nullptr;
    std::vector<int> cold_file;           // per (expert, node, piece): drive file of the piece (-1: no record)
    std::vector<long long> cold_off;      // and its byte offset there
    std::vector<float> score;
    float decay = 1.f;
    double cold_stats[4] = {0, 0, 0, 0};

    size_t gate_rows() const { return size_t(I / nodes); }
    size_t down_rows() const { return size_t(H / nodes); }
    int bs() const { return fmt == NVFP4 ? 16 : 32; }
};

static void plan_alloc(Plan *p) {
    const int N = p->nodes, bs = p->bs();
    size_t gr = p->gate_rows(), dr = p->down_rows();
    size_t sz[6] = {gr * p->H / 2, gr * p->H / 2, gr * p->H / bs, gr * p->H / bs, dr * p->I / 2, dr * p->I / bs};
    int total = p->slots + p->shared;
    for (int n = 0; n < N; ++n) {
        Shard s;
        size_t off = 0;
        for (int q = 0; q < 6; ++q) {
            s.piece_off[q] = off;
            s.piece_bytes[q] = sz[q];
            off += pad4k(sz[q]);
        }
        s.stride = off;
        s.bytes = off * size_t(std::max(total, 1));
        void *m = mmap(nullptr, s.bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
        if (m == MAP_FAILED) throw std::runtime_error("engine: mmap of the weight shard failed");
        madvise(m, s.bytes, MADV_HUGEPAGE);
        if (N > 1) {
            unsigned long mask[16] = {0};
            int node = g_topo.node_ids[n];
            mask[node / 64] |= 1ul << (node % 64);
            syscall(SYS_mbind, m, s.bytes, 2 /*MPOL_BIND*/, mask, 1024, 0);   // best effort
        }
        s.base = static_cast<uint8_t *>(m);
        p->shards.push_back(s);
    }
}

// Copies expert `src` of the input arrays into shard slot `slot`
static void plan_fill(Plan *p, int slot, int src, const uint8_t *w13, const uint8_t *w2, const uint8_t *s13,
                      const uint8_t *s2) {
    const int H = p->H, I = p->I, bs = p->bs();
    size_t gr = p->gate_rows(), dr = p->down_rows();
    for (int n = 0; n < p->nodes; ++n) {
        Shard &sh = p->shards[n];
        size_t g0 = n * gr, d0 = n * dr;
        const uint8_t *e13 = w13 + size_t(src) * 2 * I * (H / 2), *es13 = s13 + size_t(src) * 2 * I * (H / bs);
        memcpy(sh.piece(slot, 0), e13 + g0 * (H / 2), gr * (H / 2));
        memcpy(sh.piece(slot, 1), e13 + (I + g0) * (H / 2), gr * (H / 2));
        memcpy(sh.piece(slot, 2), es13 + g0 * (H / bs), gr * (H / bs));
        memcpy(sh.piece(slot, 3), es13 + (I + g0) * (H / bs), gr * (H / bs));
        memcpy(sh.piece(slot, 4), w2 + size_t(src) * H * (I / 2) + d0 * (I / 2), dr * (I / 2));
        memcpy(sh.piece(slot, 5), s2 + size_t(src) * H * (I / bs) + d0 * (I / bs), dr * (I / bs));
    }
}

// ------------------------------------------------------------------------------------------------ forward job
struct ForwardJob : Job {
    Plan *p;
    int m;
    float *y;
    std::vector<std::atomic<int>> next1, next2;
    int chunk1, chunk2, tasks1, tasks2;   // per node
    bool probe = false;
    std::atomic<long long> sink{0};
    double t_mid = 0;

    ForwardJob(Plan *p_, int m_, float *y_) : p(p_), m(m_), y(y_), next1(p_->nodes), next2(p_->nodes) {
        for (auto &a : next1) a.store(0);
        for (auto &a : next2) a.store(0);
        int workers_per_node = std::max(1, p->pool->nthreads / p->nodes);
        int ng = int(p->groups.size());
        int gr = int(p->gate_rows()), dr = int(p->down_rows());
        // about 4 tasks per worker per phase, rows a multiple of 4
        chunk1 = std::max(4, ((gr * ng) / (4 * workers_per_node) + 3) & ~3);
        chunk1 = std::min(chunk1, gr);
        chunk2 = std::max(4, (dr / (4 * workers_per_node) + 3) & ~3);
        chunk2 = std::min(chunk2, dr);
        tasks1 = ng * ((gr + chunk1 - 1) / chunk1);
        tasks2 = (dr + chunk2 - 1) / chunk2;
    }

    void run(int worker, int node) override {
        phase1(node);
        p->pool->barrier();
        if (worker == 0) t_mid = now_us();
        phase2(node);
    }

    uint8_t *xp(int t) const { return p->xprep.data() + size_t(t) * p->H * p->K->x_bytes_per_elem; }
    uint8_t *mp(int g, int j) const {
        return p->midprep.data() + (size_t(g) * MAX_TOK + j) * p->I * p->K->mid_bytes_per_elem;
    }

    void phase1(int node) {
        const Shard &sh = p->shards[node];
        const int H = p->H, bs = p->bs();
        const int gr = int(p->gate_rows());
        const int per_group = (gr + chunk1 - 1) / chunk1;
        float gate[64 * MAX_TOK], up[64 * MAX_TOK];
        for (;;) {
            int t = next1[node].fetch_add(1, std::memory_order_relaxed);
            if (t >= tasks1) break;
            const Group &g = p->groups[t / per_group];
            int r0 = (t % per_group) * chunk1, r1 = std::min(gr, r0 + chunk1);
            const void *xs[MAX_TOK];
            for (int j = 0; j < g.ntok; ++j) xs[j] = xp(g.tok[j]);
            const uint8_t *gw = sh.piece(g.slot, 0), *uw = sh.piece(g.slot, 1);
            const uint8_t *gs = sh.piece(g.slot, 2), *us = sh.piece(g.slot, 3);
            if (probe) {
                long long acc = 0;
                for (int r = r0; r < r1; ++r)
                    for (int b = 0; b < H / 2; b += 64) acc += gw[size_t(r) * H / 2 + b] + uw[size_t(r) * H / 2 + b];
                sink.fetch_add(acc, std::memory_order_relaxed);
                continue;
            }
            for (int rb = r0; rb < r1; rb += 64) {
                int rows = std::min(64, r1 - rb);
                p->K->dot(gw + size_t(rb) * (H / 2), H / 2, gs + size_t(rb) * (H / bs), H / bs, rows, H, p->fmt, xs,
                          g.ntok, 0, gate);
                p->K->dot(uw + size_t(rb) * (H / 2), H / 2, us + size_t(rb) * (H / bs), H / bs, rows, H, p->fmt, xs,
                          g.ntok, 0, up);
                for (int r = 0; r < rows; ++r)
                    for (int j = 0; j < g.ntok; ++j) {
                        float a = gate[r * g.ntok + j] * g.g_gate, u = up[r * g.ntok + j] * g.g_up;
                        if (p->limit > 0) {
                            a = std::min(a, p->limit);
                            u = std::max(-p->limit, std::min(u, p->limit));
                        }
                        float h = (p->alpha == 1.f && p->beta == 0.f)
                                      ? a / (1.f + expf(-a)) * u
                                      : a / (1.f + expf(-p->alpha * a)) * (u + p->beta);
                        p->K->store_mid(mp(int(&g - p->groups.data()), j), p->I, node * gr + rb + r, h);
                    }
            }
        }
    }

    void phase2(int node) {
        const Shard &sh = p->shards[node];
        const int I = p->I, bs = p->bs(), H = p->H;
        const int dr = int(p->down_rows());
        const int hilo = strcmp(p->K->name, "avx512") == 0;   // FP32 intermediate as an exact BF16 hi+lo pair
        float part[64 * MAX_TOK];
        for (;;) {
            int t = next2[node].fetch_add(1, std::memory_order_relaxed);
            if (t >= tasks2) break;
            int r0 = t * chunk2, r1 = std::min(dr, r0 + chunk2);
            int h0 = node * dr;
            if (!probe)
                for (int tok = 0; tok < m; ++tok) memset(y + size_t(tok) * H + h0 + r0, 0, sizeof(float) * (r1 - r0));
            for (size_t gi = 0; gi < p->groups.size(); ++gi) {
                const Group &g = p->groups[gi];
                const uint8_t *dw = sh.piece(g.slot, 4), *ds = sh.piece(g.slot, 5);
                if (probe) {
                    long long acc = 0;
                    for (int r = r0; r < r1; ++r)
                        for (int b = 0; b < I / 2; b += 64) acc += dw[size_t(r) * I / 2 + b];
                    sink.fetch_add(acc, std::memory_order_relaxed);
                    continue;
                }
                const void *xs[MAX_TOK];
                for (int j = 0; j < g.ntok; ++j) xs[j] = mp(int(gi), j);
                for (int rb = r0; rb < r1; rb += 64) {
                    int rows = std::min(64, r1 - rb);
                    p->K->dot(dw + size_t(rb) * (I / 2), I / 2, ds + size_t(rb) * (I / bs), I / bs, rows, I, p->fmt,
                              xs, g.ntok, hilo, part);
                    for (int r = 0; r < rows; ++r)
                        for (int j = 0; j < g.ntok; ++j)
                            y[size_t(g.tok[j]) * H + h0 + rb + r] += g.w[j] * g.g_down * part[r * g.ntok + j];
                }
            }
        }
    }
};

struct PrepJob : Job {   // prepares the token vectors, spread over the workers
    Plan *p;
    const uint16_t *x;
    int m;
    std::atomic<int> next{0};
    void run(int, int) override {
        for (;;) {
            int t = next.fetch_add(1);
            if (t >= m) break;
            p->K->prep_x(x + size_t(t) * p->H, p->H, p->xprep.data() + size_t(t) * p->H * p->K->x_bytes_per_elem);
        }
    }
};

static int cold_ensure(Plan *p, const std::vector<int> &need_experts, bool decode);

static int build_groups(Plan *p, int m, int k, const int32_t *ids, const float *w, bool decode, bool shared_too) {
    struct Route {
        int e, t;
        float w;
    };
    std::vector<Route> routes;
    routes.reserve(size_t(m) * k);
    std::vector<char> keep;
    bool tail = decode && p->tail_keep > 0 && k == p->tail_total && m <= p->tail_tokens;
    if (tail) {   // experts among some token's K largest routes (ties: the earlier route)
        keep.assign(p->E, 0);
        std::vector<int> order(k);
        for (int t = 0; t < m; ++t) {
            for (int j = 0; j < k; ++j) order[j] = j;
            std::stable_sort(order.begin(), order.end(),
                             [&](int a, int b) { return w[size_t(t) * k + a] > w[size_t(t) * k + b]; });
            for (int j = 0; j < p->tail_keep; ++j) {
                int e = ids[size_t(t) * k + order[j]];
                if (e >= 0 && e < p->E) keep[e] = 1;
            }
        }
    }
    std::vector<char> seen(p->E, 0);
    int distinct = 0, dropped = 0;
    for (int t = 0; t < m; ++t)
        for (int j = 0; j < k; ++j) {
            int e = ids[size_t(t) * k + j];
            if (e < 0) continue;
            if (e >= p->E) {
                set_error("engine: expert id " + std::to_string(e) + " out of range");
                return -1;
            }
            if (!seen[e]) {
                seen[e] = 1;
                ++distinct;
                if (tail && !keep[e]) ++dropped;
            }
            if (tail && !keep[e]) continue;
            routes.push_back({e, t, w[size_t(t) * k + j]});
        }
    if (tail) {
        p->tail_stats[0] += 1;
        p->tail_stats[1] += distinct;
        p->tail_stats[2] += dropped;
    }
    std::stable_sort(routes.begin(), routes.end(), [](const Route &a, const Route &b) { return a.e < b.e; });
    if (p->cold || p->slots < p->E) {
        std::vector<int> need;
        for (size_t i = 0; i < routes.size(); ++i)
            if ((i == 0 || routes[i].e != routes[i - 1].e)) need.push_back(routes[i].e);
        if (cold_ensure(p, need, decode) < 0) return -1;
    }
    p->groups.clear();
    for (size_t i = 0; i < routes.size();) {
        Group g;
        g.slot = p->slot_of[routes[i].e];
        g.ntok = 0;
        g.g_gate = p->g13[2 * g.slot];
        g.g_up = p->g13[2 * g.slot + 1];
        g.g_down = p->g2[g.slot];
        int e = routes[i].e;
        while (i < routes.size() && routes[i].e == e && g.ntok < MAX_TOK) {
            g.tok[g.ntok] = routes[i].t;
            g.w[g.ntok] = routes[i].w;
            ++g.ntok;
            ++i;
        }
        p->groups.push_back(g);
    }
    for (int s = 0; s < (shared_too ? p->shared : 0); ++s)
        for (int t0 = 0; t0 < m; t0 += MAX_TOK) {
            Group g;
            g.slot = p->slots + s;
            g.ntok = std::min(MAX_TOK, m - t0);
            for (int j = 0; j < g.ntok; ++j) {
                g.tok[j] = t0 + j;
                g.w[j] = 1.f;
            }
            g.g_gate = p->g13[2 * g.slot];
            g.g_up = p->g13[2 * g.slot + 1];
            g.g_down = p->g2[g.slot];
            p->groups.push_back(g);
        }
    return int(p->groups.size());
}

static int forward_once(Plan *p, int m, int k, const uint16_t *x, const int32_t *ids, const float *w, float *y,
                        bool decode, bool probe, bool shared_too) {
    if (p->busy.exchange(1)) {
        set_error("engine: concurrent forward on one plan");
        return -1;
    }
    std::lock_guard<std::mutex> lk(p->pool->use);
    int ng = build_groups(p, m, k, ids, w, decode, shared_too);
    if (ng < 0) {
        p->busy.store(0);
        return -1;
    }
    size_t xb = size_t(m) * p->H * p->K->x_bytes_per_elem;
    if (p->xprep.size() < xb) p->xprep.resize(xb);
    size_t mb = size_t(std::max(ng, 1)) * MAX_TOK * p->I * p->K->mid_bytes_per_elem;
    if (p->midprep.size() < mb) p->midprep.resize(mb);
    double t0 = now_us();
    if (!probe) {
        if (m <= 2) {
            for (int t = 0; t < m; ++t)
                p->K->prep_x(x + size_t(t) * p->H, p->H, p->xprep.data() + size_t(t) * p->H * p->K->x_bytes_per_elem);
        } else {
            PrepJob pj;
            pj.p = p;
            pj.x = x;
            pj.m = m;
            p->pool->run(&pj);
        }
    }
    if (ng == 0 && !probe) {
        memset(y, 0, sizeof(float) * size_t(m) * p->H);
    } else {
        ForwardJob job(p, m, y);
        job.probe = probe;
        p->pool->run(&job);
        p->t_gate = job.t_mid - t0;
        p->t_down = now_us() - job.t_mid;
    }
    p->busy.store(0);
    return ng;
}

// A call that needs more distinct experts than a cold-backed plan has unpinned RAM slots runs in batches of experts
// (ascending ids; the shared experts with the first batch), the batches' outputs summed in batch order.
static int forward_impl(Plan *p, int m, int k, const uint16_t *x, const int32_t *ids, const float *w, float *y,
                        bool decode, bool probe) {
    if (!p || m < 1 || k < 0 || (k > 0 && (!ids || !w)) || !x || (!y && !probe)) {
        set_error("engine: bad forward arguments");
        return -1;
    }
    if (p->slots >= p->E || k == 0) return forward_once(p, m, k, x, ids, w, y, decode, probe, true);
    std::vector<char> seen(p->E, 0);
    std::vector<int> need;
    for (size_t i = 0; i < size_t(m) * k; ++i) {
        const int e = ids[i];
        if (e >= 0 && e < p->E && !seen[e]) {
            seen[e] = 1;
            need.push_back(e);
        }
    }
    int cap = 0;
    for (int s = 0; s < p->slots; ++s) cap += __atomic_load_n(&p->pins[s], __ATOMIC_ACQUIRE) <= 0;
    if (int(need.size()) <= cap) return forward_once(p, m, k, x, ids, w, y, decode, probe, true);
    if (cap < 1) {
        set_error("engine: every RAM slot is pinned; no room for the call's experts");
        return -1;
    }
    std::sort(need.begin(), need.end());
    std::vector<int32_t> bids(size_t(m) * k);
    std::vector<float> part(probe ? 0 : size_t(m) * p->H);
    int total = 0;
    for (size_t b0 = 0; b0 < need.size(); b0 += size_t(cap)) {
        const int lo = need[b0], hi = need[std::min(need.size(), b0 + size_t(cap)) - 1];
        for (size_t i = 0; i < bids.size(); ++i) bids[i] = (ids[i] >= lo && ids[i] <= hi) ? ids[i] : -1;
        float *dst = (b0 == 0 || probe) ? y : part.data();
        const int ng = forward_once(p, m, k, x, bids.data(), w, dst, decode, probe, b0 == 0);
        if (ng < 0) return -1;
        total += ng;
        if (b0 > 0 && !probe)
            for (size_t i = 0; i < part.size(); ++i) y[i] += part[i];
    }
    return total;
}

// ------------------------------------------------------------------------------------------------ cold experts
}  // namespace xt

extern "C" int xt_cold_read(void *store, int jobs, const int *files, const long long *offsets, void *const *dst,
                            const size_t *sizes, int n);

namespace xt {

// The slot's global scales follow the expert that now occupies it (when per-expert scales were given).
static void slot_scales(Plan *p, int slot, int e) {
    if (p->eg13.empty()) return;
    p->g13[2 * size_t(slot)] = p->eg13[2 * size_t(e)];
    p->g13[2 * size_t(slot) + 1] = p->eg13[2 * size_t(e) + 1];
    p->g2[slot] = p->eg2[e];
}

static int cold_ensure(Plan *p, const std::vector<int> &need, bool decode) {
    for (auto &s : p->score) s *= p->decay;
    for (int e : need) p->score[e] += 1.f;
    std::vector<int> missing;
    for (int e : need)
        if (p->slot_of[e] < 0) missing.push_back(e);
    p->cold_stats[0] += 1;
    if (decode) p->cold_stats[3] += 1;
    if (missing.empty()) return 0;
    if (!p->cold) {
        set_error("engine: expert " + std::to_string(missing[0]) + " is not in RAM and no cold store is attached");
        return -1;
    }
    std::vector<char> used(p->E, 0);
    for (int e : need) used[e] = 1;
    double t0 = now_us();
    for (int e : missing) {
        if (p->cold_file[size_t(e) * p->nodes * 6] < 0) {
            set_error("engine: expert " + std::to_string(e) + " is not in RAM and has no cold record");
            return -1;
        }
        int victim = -1;
        float best = 3.4e38f;
        for (int s = 0; s < p->slots; ++s) {
            int ex = p->expert_of[s];
            if (p->pins[s] > 0) continue;
            if (ex >= 0 && used[ex]) continue;
            float sc = ex < 0 ? -1.f : p->score[ex];
            if (sc < best) {
                best = sc;
                victim = s;
            }
        }
        if (victim < 0) {
            set_error("engine: no free RAM slot for a cold expert (all slots used by this call or pinned)");
            return -1;
        }
        // every piece of every node's shard is one read job (the pieces of a record may sit on different drives)
        const int jobs = p->nodes * 6;
        std::vector<void *> dst(jobs);
        std::vector<size_t> sz(jobs);
        for (int n = 0; n < p->nodes; ++n) {
            const Shard &sh = p->shards[n];
            for (int q = 0; q < 6; ++q) {
                dst[n * 6 + q] = sh.piece(victim, q);
                sz[n * 6 + q] = (sh.piece_bytes[q] + 511) & ~size_t(511);
            }
        }
        const int *f = p->cold_file.data() + size_t(e) * jobs;
        const long long *off = p->cold_off.data() + size_t(e) * jobs;
        if (xt_cold_read(p->cold, jobs, f, off, dst.data(), sz.data(), 1) != 0) {
            set_error("engine: cold read of expert " + std::to_string(e) + " failed");
            return -1;
        }
        int old = p->expert_of[victim];
        if (old >= 0) p->slot_of[old] = -1;
        p->expert_of[victim] = e;
        p->slot_of[e] = victim;
        slot_scales(p, victim, e);
        p->cold_stats[1] += 1;
    }
    p->cold_stats[2] += (now_us() - t0) * 1e-6;
    return 0;
}

}  // namespace xt

using namespace xt;

extern "C" {

void *xt_engine_create(int hidden, int inter, int experts, int shared, int slots, int threads, float limit, int fmt,
                       const uint8_t *w13, const uint8_t *w2, const uint8_t *s13, const uint8_t *s2, const float *g13,
                       const float *g2, const int32_t *resident) {
    try {
        const Kernels *K = pick_kernels();
        if (!K) {
            set_error("engine: XTIER_ISA asks for kernels this CPU does not support");
            return nullptr;
        }
        if (fmt != NVFP4 && fmt != MXFP4) {
            set_error("engine: fmt must be 0 (NVFP4) or 1 (MXFP4)");
            return nullptr;
        }
        if (experts < 1 || shared < 0 || slots < 1 || slots > experts || hidden <= 0 || inter <= 0) {
            set_error("engine: bad shape");
            return nullptr;
        }
        Pool *pool = get_pool(threads);
        Plan *p = new Plan();
        p->H = hidden;
        p->I = inter;
        p->E = experts;
        p->shared = shared;
        p->slots = slots;
        p->fmt = fmt;
        p->limit = limit;
        p->K = K;
        p->pool = pool;
        p->nodes = pool->nnodes;
        while (p->nodes > 1 && ((hidden / p->nodes) % 4 || (inter / p->nodes) % 4 || hidden % p->nodes ||
                                inter % p->nodes))
            --p->nodes;   // rows must split evenly; fewer shards otherwise
        if (hidden % K->chunk || inter % K->chunk) {
            set_error("engine: hidden and inter must be multiples of " + std::to_string(K->chunk) + " for the " +
                      K->name + " kernels");
            delete p;
            return nullptr;
        }
        plan_alloc(p);
        int total = slots + shared;
        p->g13.assign(size_t(total) * 2, 1.f);
        p->g2.assign(total, 1.f);
        p->slot_of.assign(experts, -1);
        p->expert_of.assign(slots, -1);
        p->pins.assign(slots, 0);
        p->score.assign(experts, 0.f);
        for (int s = 0; s < slots; ++s) {
            int e = resident ? resident[s] : (w13 ? s : -1);   // unfilled slots hold no expert unless named
            if (e >= 0 && e < experts) {
                p->expert_of[s] = e;
                p->slot_of[e] = s;
            }
        }
        if (w13) {
            for (int s = 0; s < total; ++s) plan_fill(p, s, s, w13, w2, s13, s2);
        }
        if (g13)
            for (int s = 0; s < total; ++s) {
                p->g13[2 * s] = g13[2 * s];
                p->g13[2 * s + 1] = g13[2 * s + 1];
                p->g2[s] = g2[s];
            }
        const char *ts = getenv("XTIER_TAIL_SKIP");
        if (ts && *ts && strcmp(ts, "0") != 0) {
            int a = 0, b = 0;
            if (sscanf(ts, "%d/%d", &a, &b) != 2 || a < 1 || b < a) {
                set_error(std::string("engine: XTIER_TAIL_SKIP must be K/N, got ") + ts);
                delete p;
                return nullptr;
            }
            p->tail_keep = a;
            p->tail_total = b;
        }
        p->tail_tokens = env_int("XTIER_TAIL_SKIP_TOKENS", 8);
        return p;
    } catch (const std::exception &e) {
        set_error(e.what());
        return nullptr;
    }
}

void xt_engine_destroy(void *plan) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p) return;
    for (auto &s : p->shards) munmap(s.base, s.bytes);
    delete p;
}

int xt_engine_set_swiglu(void *plan, float alpha, float beta) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p) return -1;
    p->alpha = alpha;
    p->beta = beta;
    return 0;
}

int xt_engine_forward(void *plan, int m, int k, const uint16_t *x, const int32_t *ids, const float *w, float *y) {
    return forward_impl(static_cast<Plan *>(plan), m, k, x, ids, w, y, false, false);
}

int xt_engine_forward_decode(void *plan, int m, int k, const uint16_t *x, const int32_t *ids, const float *w,
                             float *y) {
    return forward_impl(static_cast<Plan *>(plan), m, k, x, ids, w, y, true, false);
}

int xt_engine_read_probe(void *plan, int m, int k, const int32_t *ids) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p) return -1;
    std::vector<float> w(size_t(m) * k, 1.f);
    std::vector<uint16_t> x(size_t(m) * p->H, 0);
    return forward_impl(p, m, k, x.data(), ids, w.data(), nullptr, false, true);
}

int xt_engine_shape(void *plan, int *o) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p) return -1;
    o[0] = p->H;
    o[1] = p->I;
    o[2] = p->E;
    o[3] = p->shared;
    o[4] = p->slots;
    o[5] = p->nodes;
    o[6] = p->pool->nthreads;
    return 0;
}

void xt_engine_last_timings(void *plan, double *o) {
    Plan *p = static_cast<Plan *>(plan);
    o[0] = p ? p->t_gate : 0;
    o[1] = p ? p->t_down : 0;
}

void xt_engine_tail_stats(void *plan, double *o) {
    Plan *p = static_cast<Plan *>(plan);
    for (int i = 0; i < 3; ++i) o[i] = p ? p->tail_stats[i] : 0;
}

int xt_engine_slot_table(void *plan, int32_t *table) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p) return -1;
    for (int e = 0; e < p->E; ++e) table[e] = p->slot_of[e];
    return p->slots;
}

int xt_engine_place(void *plan, int expert, int slot) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p || expert < -1 || expert >= p->E || slot < 0 || slot >= p->slots) return -2;
    if (p->busy.load()) return -3;
    int old = p->expert_of[slot];
    if (old >= 0) p->slot_of[old] = -1;
    if (expert < 0) {          // vacate the slot
        p->expert_of[slot] = -1;
        return old;
    }
    int prev = p->slot_of[expert];
    if (prev >= 0) p->expert_of[prev] = -1;
    p->expert_of[slot] = expert;
    p->slot_of[expert] = slot;
    slot_scales(p, slot, expert);
    return old;
}

int xt_engine_expert_scales(void *plan, const float *g13, const float *g2) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p || !g13 || !g2) return -1;
    if (p->busy.load()) return -3;
    p->eg13.assign(g13, g13 + size_t(p->E) * 2);
    p->eg2.assign(g2, g2 + p->E);
    for (int s = 0; s < p->slots; ++s)
        if (p->expert_of[s] >= 0) slot_scales(p, s, p->expert_of[s]);
    return 0;
}

int xt_engine_slot_pin(void *plan, int expert) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p || expert < 0 || expert >= p->E) return -1;
    int s = p->slot_of[expert];
    if (s >= 0) __atomic_add_fetch(&p->pins[s], 1, __ATOMIC_ACQ_REL);
    return s;
}

void xt_engine_slot_unpin(void *plan, int slot) {
    Plan *p = static_cast<Plan *>(plan);
    if (p && slot >= 0 && slot < p->slots) __atomic_sub_fetch(&p->pins[slot], 1, __ATOMIC_ACQ_REL);
}

int xt_engine_slot_pieces(void *plan, int slot, int node, void **ptrs, size_t *bytes) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p || slot < 0 || slot >= p->slots + p->shared || node < 0 || node >= p->nodes) return -1;
    for (int q = 0; q < 6; ++q) {
        ptrs[q] = p->shards[node].piece(slot, q);
        bytes[q] = p->shards[node].piece_bytes[q];
    }
    return 0;
}

int xt_engine_shard(void *plan, int node, void **base, size_t *bytes, size_t *stride, size_t *piece_off,
                    size_t *piece_bytes) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p || node < 0 || node >= p->nodes) return -1;
    const Shard &s = p->shards[node];
    *base = s.base;
    *bytes = s.bytes;
    *stride = s.stride;
    for (int q = 0; q < 6; ++q) {
        piece_off[q] = s.piece_off[q];
        piece_bytes[q] = s.piece_bytes[q];
    }
    return 0;
}

int xt_engine_nodes(void *plan) {
    Plan *p = static_cast<Plan *>(plan);
    return p ? p->nodes : -1;
}

int xt_engine_cold_attach_pieces(void *plan, void *store, const int32_t *files, const long long *offsets,
                                 const float *scores, float half_life) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p || !store) return -1;
    p->cold = store;
    p->cold_file.assign(files, files + size_t(p->E) * p->nodes * 6);
    p->cold_off.assign(offsets, offsets + size_t(p->E) * p->nodes * 6);
    if (scores) p->score.assign(scores, scores + p->E);
    p->decay = half_life > 0 ? powf(0.5f, 1.f / half_life) : 1.f;
    return 0;
}

// Whole records: the six pieces of (expert, node) follow each other from the record's offset, each padded to 512 B.
int xt_engine_cold_attach(void *plan, void *store, const int32_t *files, const long long *offsets, const float *scores,
                          float half_life) {
    Plan *p = static_cast<Plan *>(plan);
    if (!p || !store) return -1;
    const size_t recs = size_t(p->E) * p->nodes;
    std::vector<int32_t> pf(recs * 6);
    std::vector<long long> po(recs * 6);
    for (size_t r = 0; r < recs; ++r) {
        const Shard &sh = p->shards[r % p->nodes];
        long long o = offsets[r];
        for (int q = 0; q < 6; ++q) {
            pf[r * 6 + q] = files[r];
            po[r * 6 + q] = o;
            o += (long long)((sh.piece_bytes[q] + 511) & ~size_t(511));
        }
    }
    return xt_engine_cold_attach_pieces(plan, store, pf.data(), po.data(), scores, half_life);
}

void xt_engine_cold_stats(void *plan, double *o) {
    Plan *p = static_cast<Plan *>(plan);
    for (int i = 0; i < 4; ++i) o[i] = p ? p->cold_stats[i] : 0;
}

int xt_engine_worker_cpus(int threads, int *cpus, int capacity) {
    Topology t = read_topology();
    auto w = worker_cpus(t, threads);
    int n = 0;
    for (auto &v : w)
        for (int c : v)
            if (n < capacity) cpus[n++] = c;
    return n;
}

const char *xt_engine_isa(void) {
    const Kernels *k = pick_kernels();
    return k ? k->name : "none";
}

const char *xt_engine_error(void) { return g_error.c_str(); }

}  // extern "C"
