// Cold-expert store: expert records on NVMe files (one per drive), read and written with O_DIRECT so nothing passes
// the page cache. Each file has its own reader threads and job queue; synchronous reads (a decode forward waiting for
// its experts) are queued ahead of asynchronous tickets (a prefill's read-ahead). A ticket counts its jobs per group so
// a caller can wait for the first experts while later ones are still in flight.
// Reference parity: csrc/cold/store.cpp (xtier_cold_open/write/read/submit/wait/finish/stats/close); the queueing and
// ticket design here are this project's own.
#include "../include/xt_engine.h"

#include <errno.h>
#include <fcntl.h>
#include <limits.h>
#include <stdlib.h>
#include <string.h>
#include <sys/uio.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_err;

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

struct Ticket {
    std::mutex mu;
    std::condition_variable cv;
    std::vector<int> remaining;   // per group
    int total = 0;
    bool failed = false;
    double t_submit = 0;
};

struct ReadJob {
    Ticket *ticket;
    int group;
    long long offset;
    std::vector<iovec> iov;
};

struct File {
    int fd = -1;
    std::mutex mu;
    std::condition_variable cv;
    std::deque<ReadJob> queue;
    std::vector<std::thread> readers;
};

struct Store {
    std::vector<std::unique_ptr<File>> files;
    bool stop = false;
    std::atomic<long long> bytes_read{0}, bytes_written{0}, jobs{0};
    std::mutex stat_mu;
    double seconds = 0;
};

void finish_job(Store *s, ReadJob &j, bool ok) {
    std::lock_guard<std::mutex> lk(j.ticket->mu);
    if (!ok) j.ticket->failed = true;
    --j.ticket->remaining[j.group];
    --j.ticket->total;
    j.ticket->cv.notify_all();
    (void)s;
}

void reader(Store *s, File *f) {
    for (;;) {
        ReadJob j;
        {
            std::unique_lock<std::mutex> lk(f->mu);
            f->cv.wait(lk, [&] { return s->stop || !f->queue.empty(); });
            if (f->queue.empty()) return;
            j = std::move(f->queue.front());
            f->queue.pop_front();
        }
        bool ok = true;
        long long off = j.offset;
        size_t idx = 0;
        std::vector<iovec> iov = j.iov;
        while (idx < iov.size()) {
            ssize_t n = preadv(f->fd, iov.data() + idx, int(std::min<size_t>(iov.size() - idx, IOV_MAX)), off);
            if (n < 0 && errno == EINTR) continue;
            if (n <= 0) {
                ok = false;
                break;
            }
            s->bytes_read += n;
            off += n;
            while (n > 0 && idx < iov.size()) {
                if (size_t(n) >= iov[idx].iov_len) {
                    n -= iov[idx].iov_len;
                    ++idx;
                } else {
                    iov[idx].iov_base = static_cast<char *>(iov[idx].iov_base) + n;
                    iov[idx].iov_len -= n;
                    n = 0;
                }
            }
        }
        s->jobs += 1;
        finish_job(s, j, ok);
    }
}

bool aligned512(const void *p, size_t n) { return (reinterpret_cast<uintptr_t>(p) % 512) == 0 && n % 512 == 0; }

Ticket *submit(Store *s, int jobs, const int *files, const long long *offsets, void *const *dst, const size_t *sizes,
               int n, const int *groups, int group_count, bool front) {
    auto *t = new Ticket();
    t->remaining.assign(std::max(group_count, 1), 0);
    t->t_submit = now_s();
    std::vector<std::pair<File *, ReadJob>> todo;
    for (int j = 0; j < jobs; ++j) {
        if (files[j] < 0 || files[j] >= int(s->files.size()) || offsets[j] % 512) {
            g_err = "cold store: bad file index or unaligned offset";
            delete t;
            return nullptr;
        }
        ReadJob r;
        r.ticket = t;
        r.group = groups ? groups[j] : 0;
        if (r.group < 0 || r.group >= int(t->remaining.size())) {
            g_err = "cold store: bad group";
            delete t;
            return nullptr;
        }
        r.offset = offsets[j];
        for (int q = 0; q < n; ++q) {
            void *d = dst[size_t(j) * n + q];
            size_t sz = sizes[size_t(j) * n + q];
            if (!aligned512(d, sz)) {
                g_err = "cold store: read buffers and sizes must be 512-byte aligned";
                delete t;
                return nullptr;
            }
            r.iov.push_back({d, sz});
        }
        t->remaining[r.group]++;
        t->total++;
        todo.emplace_back(s->files[files[j]].get(), std::move(r));
    }
    for (auto &fj : todo) {
        std::lock_guard<std::mutex> lk(fj.first->mu);
        if (front)
            fj.first->queue.push_front(std::move(fj.second));
        else
            fj.first->queue.push_back(std::move(fj.second));
        fj.first->cv.notify_one();
    }
    return t;
}

int wait_groups(Ticket *t, int g0, int g1) {
    std::unique_lock<std::mutex> lk(t->mu);
    t->cv.wait(lk, [&] {
        for (int g = g0; g < g1; ++g)
            if (t->remaining[g] > 0) return false;
        return true;
    });
    return t->failed ? -1 : 0;
}

}  // namespace

extern "C" {

void *xt_cold_open(const char *const *paths, int count, int threads, int writable) {
    if (count < 1 || !paths) {
        g_err = "cold store: no files";
        return nullptr;
    }
    auto *s = new Store();
    for (int i = 0; i < count; ++i) {
        auto f = std::make_unique<File>();
        int flags = (writable ? O_RDWR | O_CREAT : O_RDONLY);
        f->fd = open(paths[i], flags | O_DIRECT, 0644);
        if (f->fd < 0) f->fd = open(paths[i], flags, 0644);   // tmpfs and friends have no O_DIRECT
        if (f->fd < 0) {
            g_err = std::string("cold store: cannot open ") + paths[i] + ": " + strerror(errno);
            for (auto &g : s->files) close(g->fd);
            delete s;
            return nullptr;
        }
        s->files.push_back(std::move(f));
    }
    for (auto &f : s->files)
        for (int t = 0; t < std::max(1, threads); ++t) f->readers.emplace_back(reader, s, f.get());
    return s;
}

int xt_cold_write(void *store, int file, long long offset, const void *const *pieces, const size_t *sizes, int n) {
    auto *s = static_cast<Store *>(store);
    if (!s || file < 0 || file >= int(s->files.size()) || offset % 512) return -1;
    size_t total = 0;
    for (int q = 0; q < n; ++q) total += (sizes[q] + 511) & ~size_t(511);
    void *buf = nullptr;
    if (posix_memalign(&buf, 4096, total ? total : 512)) return -1;
    memset(buf, 0, total);
    size_t o = 0;
    for (int q = 0; q < n; ++q) {
        memcpy(static_cast<char *>(buf) + o, pieces[q], sizes[q]);
        o += (sizes[q] + 511) & ~size_t(511);
    }
    size_t done = 0;
    int rc = 0;
    while (done < total) {
        ssize_t w = pwrite(s->files[file]->fd, static_cast<char *>(buf) + done, total - done, offset + done);
        if (w < 0 && errno == EINTR) continue;
        if (w <= 0) {
            g_err = std::string("cold store: write failed: ") + strerror(errno);
            rc = -1;
            break;
        }
        done += w;
    }
    if (rc == 0 && fdatasync(s->files[file]->fd) != 0) rc = -1;
    s->bytes_written += done;
    free(buf);
    return rc;
}

int xt_cold_read(void *store, int jobs, const int *files, const long long *offsets, void *const *dst,
                 const size_t *sizes, int n) {
    auto *s = static_cast<Store *>(store);
    if (!s) return -1;
    Ticket *t = submit(s, jobs, files, offsets, dst, sizes, n, nullptr, 1, true);
    if (!t) return -1;
    int rc = wait_groups(t, 0, 1);
    {
        std::lock_guard<std::mutex> lk(s->stat_mu);
        s->seconds += now_s() - t->t_submit;
    }
    delete t;
    return rc;
}

void *xt_cold_submit(void *store, int jobs, const int *files, const long long *offsets, void *const *dst,
                     const size_t *sizes, int n, const int *groups, int group_count) {
    auto *s = static_cast<Store *>(store);
    if (!s) return nullptr;
    return submit(s, jobs, files, offsets, dst, sizes, n, groups, group_count, false);
}

int xt_cold_wait(void *store, void *ticket, int g0, int g1) {
    (void)store;
    auto *t = static_cast<Ticket *>(ticket);
    if (!t || g0 < 0 || g1 > int(t->remaining.size()) || g0 > g1) return -1;
    return wait_groups(t, g0, g1);
}

int xt_cold_finish(void *store, void *ticket) {
    auto *s = static_cast<Store *>(store);
    auto *t = static_cast<Ticket *>(ticket);
    if (!t) return -1;
    int rc = wait_groups(t, 0, int(t->remaining.size()));
    if (s) {
        std::lock_guard<std::mutex> lk(s->stat_mu);
        s->seconds += now_s() - t->t_submit;
    }
    delete t;
    return rc;
}

void xt_cold_stats(void *store, double *o) {
    auto *s = static_cast<Store *>(store);
    if (!s) return;
    o[0] = double(s->bytes_read.load());
    o[1] = double(s->bytes_written.load());
    o[2] = double(s->jobs.load());
    std::lock_guard<std::mutex> lk(s->stat_mu);
    o[3] = s->seconds;
}

void xt_cold_close(void *store) {
    auto *s = static_cast<Store *>(store);
    if (!s) return;
    for (auto &f : s->files) {
        {
            std::lock_guard<std::mutex> lk(f->mu);
            s->stop = true;
        }
        f->cv.notify_all();
    }
    for (auto &f : s->files)
        for (auto &t : f->readers) t.join();
    for (auto &f : s->files) close(f->fd);
    delete s;
}

const char *xt_cold_error(void) { return g_err.c_str(); }

}  // extern "C"
