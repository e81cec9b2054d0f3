/* Minimal hls::stream<T> for compiling the reference's native decode model.
 *
 * TEST INFRASTRUCTURE ONLY (oracle/Makefile). Semantics the reference relies
 * on: an unbounded FIFO; read() blocks until data arrives (the reference
 * builds with HLS_STREAM_THREAD_SAFE, and its partitioned model runs three
 * kernels as threads over these streams); read_nb/write_nb never block;
 * write_nb always succeeds because the FIFO is unbounded. A read that stays
 * empty for a long time aborts with the stream's name instead of hanging.
 */
#ifndef GDN_SHIM_HLS_STREAM_H
#define GDN_SHIM_HLS_STREAM_H

#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <deque>
#include <mutex>
#include <string>

namespace hls {

template <typename T> class stream {
  public:
    stream() : name_("hls::stream") {}
    explicit stream(const char *name) : name_(name ? name : "hls::stream") {}
    stream(const stream &) = delete;
    stream &operator=(const stream &) = delete;

    void write(const T &value) {
        {
            std::lock_guard<std::mutex> lock(m_);
            q_.push_back(value);
        }
        cv_.notify_one();
    }
    bool write_nb(const T &value) {
        write(value);
        return true;
    }
    T read() {
        std::unique_lock<std::mutex> lock(m_);
        if (q_.empty()) {
            if (!cv_.wait_for(lock, std::chrono::seconds(30), [this] { return !q_.empty(); })) {
                std::fprintf(stderr, "hls shim: read of empty stream '%s' did not complete\n",
                             name_.c_str());
                std::abort();
            }
        }
        T value = q_.front();
        q_.pop_front();
        return value;
    }
    void read(T &value) { value = read(); }
    bool read_nb(T &value) {
        std::lock_guard<std::mutex> lock(m_);
        if (q_.empty()) return false;
        value = q_.front();
        q_.pop_front();
        return true;
    }
    bool empty() const {
        std::lock_guard<std::mutex> lock(m_);
        return q_.empty();
    }
    bool full() const { return false; }
    size_t size() const {
        std::lock_guard<std::mutex> lock(m_);
        return q_.size();
    }
    stream &operator<<(const T &value) {
        write(value);
        return *this;
    }
    stream &operator>>(T &value) {
        value = read();
        return *this;
    }

  private:
    std::string name_;
    std::deque<T> q_;
    mutable std::mutex m_;
    std::condition_variable cv_;
};

}  // namespace hls

#endif
