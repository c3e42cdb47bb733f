// NVMe row tables: a [rows, row_bytes] table (optionally with per-row scale bytes) stored as segments in files, looked
// up by row id from a CUDA-graph host node (cudaLaunchHostFunc) or a host thread. The lookup calls no CUDA API.
//
//  * Layout: segment s covers rows [first[s], first[s] + count[s]) and lives in file path[s] at byte offset off[s],
//    rows contiguous (row_bytes each), then optionally the segment's scales (scale_bytes per row) at soff[s].
//  * Direct mode (default): the misses of one lookup are deduplicated per 4 KiB page, sorted by file and offset, merged
//    into runs and read with O_DIRECT by an IO thread pool in rounds of at most 16384 pages, into an aligned bounce
//    buffer; the rows are then copied out (and into the cache).
//  * Row cache: direct-mapped, `cache_rows` entries, tag = row id.
//  * RAM mode: every segment is mapped (and locked when allowed); lookups are copies.
//  * TP range: rows outside [lo, hi) read as zeros (a rank holding a slice of the table).
//  * An id outside the table fails the lookup (returns -1; the error text says which id); a failed read likewise.
// Reference parity: csrc/tables/rows.cpp (xtier_rows_open/lookup/prefetch/preload_scales/range/stats/close); the
// implementation here is this project's own.
#include <errno.h>
#include <fcntl.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_err;
constexpr size_t PAGE = 4096;
constexpr size_t MAX_ROUND_PAGES = 16384;
constexpr long long PGL = 4096;

struct Segment {
    std::string path;
    int fd = -1;
    long long first = 0, count = 0;
    long long off = 0, soff = -1;
    uint8_t *map = nullptr;   // RAM mode
    size_t map_bytes = 0;
};

class IoPool {
  public:
    explicit IoPool(int n) {
        for (int i = 0; i < n; ++i) threads_.emplace_back([this] { loop(); });
    }
    ~IoPool() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto &t : threads_) t.join();
    }
    // runs all tasks, returns when every one finished
    void run(std::vector<std::function<void()>> &tasks) {
        std::atomic<size_t> left{tasks.size()};
        std::mutex dm;
        std::condition_variable dcv;
        {
            std::lock_guard<std::mutex> lk(mu_);
            for (auto &t : tasks)
                queue_.push_back([&, t] {
                    t();
                    if (left.fetch_sub(1) == 1) {
                        std::lock_guard<std::mutex> l2(dm);
                        dcv.notify_all();
                    }
                });
        }
        cv_.notify_all();
        std::unique_lock<std::mutex> lk(dm);
        dcv.wait(lk, [&] { return left.load() == 0; });
    }

  private:
    std::vector<std::thread> threads_;
    std::vector<std::function<void()>> queue_;
    std::mutex mu_;
    std::condition_variable cv_;
    bool stop_ = false;
    void loop() {
        for (;;) {
            std::function<void()> f;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return stop_ || !queue_.empty(); });
                if (queue_.empty()) return;
                f = std::move(queue_.back());
                queue_.pop_back();
            }
            f();
        }
    }
};

struct Table {
    std::vector<Segment> segs;
    long long rows = 0, row_bytes = 0, scale_bytes = 0;
    long long lo = 0, hi = -1;   // TP range; hi < 0: everything
    bool ram = false;
    std::unique_ptr<IoPool> io;
    // cache
    size_t cache_rows = 0;
    std::vector<long long> tag;
    std::vector<uint8_t> cache;
    std::mutex mu;
    double stats[6] = {0, 0, 0, 0, 0, 0};   // lookups, rows, hits, misses, pages read, bytes read

    int seg_of(long long id) const {
        int a = 0, b = int(segs.size()) - 1;
        while (a <= b) {
            int m = (a + b) / 2;
            if (id < segs[m].first)
                b = m - 1;
            else if (id >= segs[m].first + segs[m].count)
                a = m + 1;
            else
                return m;
        }
        return -1;
    }
    size_t entry_bytes() const { return size_t(row_bytes + scale_bytes); }
};

bool read_full(int fd, void *dst, size_t n, off_t off) {
    size_t done = 0;
    while (done < n) {
        ssize_t r = pread(fd, static_cast<char *>(dst) + done, n - done, off + done);
        if (r < 0 && errno == EINTR) continue;
        if (r < 0) return false;
        if (r == 0) {   // end of file inside the last page: the rest of the page is not table data
            memset(static_cast<char *>(dst) + done, 0, n - done);
            return true;
        }
        done += size_t(r);
    }
    return true;
}

}  // namespace

extern "C" {

// paths/first/count/off/soff: nseg segments. mode 0 direct, 1 ram. Returns NULL on error (xt_rows_error).
void *xt_rows_open(const char *const *paths, const long long *first, const long long *count, const long long *off,
                   const long long *soff, int nseg, long long row_bytes, long long scale_bytes, int io_threads,
                   long long cache_rows, int mode) {
    auto *t = new Table();
    t->row_bytes = row_bytes;
    t->scale_bytes = scale_bytes;
    t->ram = mode == 1;
    for (int s = 0; s < nseg; ++s) {
        Segment g;
        g.path = paths[s];
        g.first = first[s];
        g.count = count[s];
        g.off = off[s];
        g.soff = soff ? soff[s] : -1;
        g.fd = open(paths[s], O_RDONLY | (t->ram ? 0 : O_DIRECT));
        if (g.fd < 0 && !t->ram) g.fd = open(paths[s], O_RDONLY);   // filesystems without O_DIRECT
        if (g.fd < 0) {
            g_err = std::string("rows: cannot open ") + paths[s] + ": " + strerror(errno);
            for (auto &x : t->segs) close(x.fd);
            delete t;
            return nullptr;
        }
        if (t->ram) {
            struct stat st;
            fstat(g.fd, &st);
            g.map_bytes = size_t(st.st_size);
            void *m = mmap(nullptr, g.map_bytes, PROT_READ, MAP_SHARED | MAP_POPULATE, g.fd, 0);
            if (m == MAP_FAILED) {
                g_err = "rows: mmap failed";
                delete t;
                return nullptr;
            }
            mlock(m, g.map_bytes);   // best effort
            g.map = static_cast<uint8_t *>(m);
        }
        t->segs.push_back(g);
        t->rows = std::max(t->rows, g.first + g.count);
    }
    std::sort(t->segs.begin(), t->segs.end(), [](const Segment &a, const Segment &b) { return a.first < b.first; });
    t->io = std::make_unique<IoPool>(std::max(1, io_threads));
    t->cache_rows = size_t(std::max(0LL, cache_rows));
    t->tag.assign(t->cache_rows, -1);
    t->cache.resize(t->cache_rows * t->entry_bytes());
    return t;
}

int xt_rows_range(void *h, long long lo, long long hi) {
    auto *t = static_cast<Table *>(h);
    if (!t) return -1;
    t->lo = lo;
    t->hi = hi;
    return 0;
}

// rows_out [n, row_bytes], scales_out [n, scale_bytes] (may be NULL). 0 or -1.
int xt_rows_lookup(void *h, const long long *ids, int n, void *rows_out, void *scales_out) {
    auto *t = static_cast<Table *>(h);
    if (!t) return -1;
    std::lock_guard<std::mutex> lk(t->mu);
    const size_t rb = size_t(t->row_bytes), sb = size_t(t->scale_bytes);
    uint8_t *ro = static_cast<uint8_t *>(rows_out);
    uint8_t *so = static_cast<uint8_t *>(scales_out);
    t->stats[0] += 1;
    t->stats[1] += n;
    struct Miss {
        int idx;
        long long id;
        int seg;
    };
    std::vector<Miss> misses;
    for (int i = 0; i < n; ++i) {
        const long long id = ids[i];
        if (id < 0 || id >= t->rows) {
            g_err = "rows: id " + std::to_string(id) + " outside the table";
            return -1;
        }
        if (t->hi >= 0 && (id < t->lo || id >= t->hi)) {   // another rank's rows
            memset(ro + size_t(i) * rb, 0, rb);
            if (so) memset(so + size_t(i) * sb, 0, sb);
            continue;
        }
        const int s = t->seg_of(id);
        if (s < 0) {
            g_err = "rows: id " + std::to_string(id) + " in no segment";
            return -1;
        }
        const Segment &g = t->segs[s];
        if (t->ram) {
            memcpy(ro + size_t(i) * rb, g.map + g.off + (id - g.first) * rb, rb);
            if (so && sb) memcpy(so + size_t(i) * sb, g.map + g.soff + (id - g.first) * sb, sb);
            continue;
        }
        if (t->cache_rows) {
            size_t c = size_t(id) % t->cache_rows;
            if (t->tag[c] == id) {
                memcpy(ro + size_t(i) * rb, &t->cache[c * t->entry_bytes()], rb);
                if (so && sb) memcpy(so + size_t(i) * sb, &t->cache[c * t->entry_bytes() + rb], sb);
                t->stats[2] += 1;
                continue;
            }
        }
        misses.push_back({i, id, s});
    }
    if (misses.empty() || t->ram) return 0;
    t->stats[3] += double(misses.size());
    // pages to read: (segment, page index in file) for the row bytes and the scale bytes of every miss
    struct Page {
        int seg;
        long long page;
    };
    std::vector<Page> pages;
    auto add_range = [&](int s, long long byte0, long long bytes) {
        for (long long p = byte0 / PGL; p <= (byte0 + bytes - 1) / PGL; ++p) pages.push_back({s, p});
    };
    for (auto &m : misses) {
        const Segment &g = t->segs[m.seg];
        add_range(m.seg, g.off + (m.id - g.first) * t->row_bytes, t->row_bytes);
        if (sb && g.soff >= 0) add_range(m.seg, g.soff + (m.id - g.first) * t->scale_bytes, t->scale_bytes);
    }
    std::sort(pages.begin(), pages.end(),
              [](const Page &a, const Page &b) { return a.seg != b.seg ? a.seg < b.seg : a.page < b.page; });
    pages.erase(std::unique(pages.begin(), pages.end(),
                            [](const Page &a, const Page &b) { return a.seg == b.seg && a.page == b.page; }),
                pages.end());
    t->stats[4] += double(pages.size());
    std::vector<int> ok(1, 1);
    for (size_t r0 = 0; r0 < pages.size(); r0 += MAX_ROUND_PAGES) {
        const size_t r1 = std::min(pages.size(), r0 + MAX_ROUND_PAGES);
        void *bounce = nullptr;
        if (posix_memalign(&bounce, PAGE, (r1 - r0) * PAGE)) return -1;
        uint8_t *bb = static_cast<uint8_t *>(bounce);
        // runs of consecutive pages of one segment
        std::vector<std::function<void()>> tasks;
        std::atomic<int> failed{0};
        size_t a = r0;
        while (a < r1) {
            size_t b = a + 1;
            while (b < r1 && pages[b].seg == pages[a].seg && pages[b].page == pages[b - 1].page + 1 && b - a < 256) ++b;
            const int fd = t->segs[pages[a].seg].fd;
            const off_t off = off_t(pages[a].page) * PAGE;
            uint8_t *dst = bb + (a - r0) * PAGE;
            const size_t bytes = (b - a) * PAGE;
            tasks.push_back([fd, off, dst, bytes, &failed] {
                if (!read_full(fd, dst, bytes, off)) failed.fetch_add(1);
            });
            a = b;
        }
        t->io->run(tasks);
        if (failed.load()) {
            free(bounce);
            g_err = "rows: a read failed";
            return -1;
        }
        t->stats[5] += double((r1 - r0) * PAGE);
        // copy out every miss whose bytes lie in this round
        auto find_page = [&](int s, long long p) -> const uint8_t * {
            auto it = std::lower_bound(pages.begin() + r0, pages.begin() + r1, Page{s, p}, [](const Page &x, const Page &y) {
                return x.seg != y.seg ? x.seg < y.seg : x.page < y.page;
            });
            if (it == pages.begin() + r1 || it->seg != s || it->page != p) return nullptr;
            return bb + size_t(it - (pages.begin() + r0)) * PAGE;
        };
        auto copy_bytes = [&](int s, long long byte0, long long bytes, uint8_t *dst) {
            for (long long done = 0; done < bytes;) {
                const long long pos = byte0 + done;
                const uint8_t *src = find_page(s, pos / PGL);
                const long long in_page = std::min(bytes - done, PGL - pos % PGL);
                if (src) memcpy(dst + done, src + pos % PGL, size_t(in_page));
                done += in_page;
            }
        };
        for (auto &m : misses) {
            const Segment &g = t->segs[m.seg];
            const long long rbyte = g.off + (m.id - g.first) * t->row_bytes;
            if (find_page(m.seg, rbyte / PGL))
                copy_bytes(m.seg, rbyte, t->row_bytes, ro + size_t(m.idx) * rb);
            if (so && sb && g.soff >= 0) {
                const long long sbyte = g.soff + (m.id - g.first) * t->scale_bytes;
                if (find_page(m.seg, sbyte / PGL))
                    copy_bytes(m.seg, sbyte, t->scale_bytes, so + size_t(m.idx) * sb);
            }
        }
        free(bounce);
    }
    if (t->cache_rows)
        for (auto &m : misses) {
            size_t c = size_t(m.id) % t->cache_rows;
            t->tag[c] = m.id;
            memcpy(&t->cache[c * t->entry_bytes()], ro + size_t(m.idx) * rb, rb);
            if (so && sb) memcpy(&t->cache[c * t->entry_bytes() + rb], so + size_t(m.idx) * sb, sb);
        }
    return 0;
}

// Warms the cache with `ids` (no output).
int xt_rows_prefetch(void *h, const long long *ids, int n) {
    auto *t = static_cast<Table *>(h);
    if (!t) return -1;
    std::vector<uint8_t> rows(size_t(n) * t->row_bytes), sc(size_t(n) * std::max(1LL, t->scale_bytes));
    return xt_rows_lookup(h, ids, n, rows.data(), t->scale_bytes ? sc.data() : nullptr);
}

// out[6]: lookups, rows, cache hits, misses, pages read, bytes read
void xt_rows_stats(void *h, double *out) {
    auto *t = static_cast<Table *>(h);
    if (!t) return;
    std::lock_guard<std::mutex> lk(t->mu);
    for (int i = 0; i < 6; ++i) out[i] = t->stats[i];
}

void xt_rows_close(void *h) {
    auto *t = static_cast<Table *>(h);
    if (!t) return;
    for (auto &g : t->segs) {
        if (g.map) munmap(g.map, g.map_bytes);
        close(g.fd);
    }
    delete t;
}

const char *xt_rows_error(void) { return g_err.c_str(); }

// Graph-capturable lookup: a CUDA host-function node calls this with a context the caller keeps alive. The ids were
// copied into pinned host memory by the node before it; the rows land in pinned host memory for the copy node after
// it. A failed lookup leaves zero rows and sets ctx->error (the caller checks it between replays); nothing here calls
// CUDA, as a host node must not.
struct XtRowsGraphCtx {
    void *store;
    const long long *ids;
    int n;
    void *rows;
    void *scales;
    volatile int error;
};

void xt_rows_host_fn(void *arg) {
    auto *c = static_cast<XtRowsGraphCtx *>(arg);
    if (xt_rows_lookup(c->store, c->ids, c->n, c->rows, c->scales) != 0) c->error = 1;
}

}  // extern "C"
