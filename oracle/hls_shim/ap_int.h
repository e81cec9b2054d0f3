/* Minimal arbitrary-width unsigned integer for compiling the reference's
 * native (csim) decode model on a machine without the Xilinx HLS headers.
 *
 * TEST INFRASTRUCTURE ONLY: used by oracle/Makefile to build the reference
 * c_impl/gdn_model.cpp as the parity oracle. Written from the documented
 * behaviour of ap_uint<N> that the reference relies on (value semantics,
 * bit and range selection as rvalue and lvalue, little-endian packing of the
 * storage so memcpy lane access works, sizeof(ap_uint<512>) == 64); it is
 * not a general replacement.
 *
 * Widths up to 64 bits convert implicitly to unsigned long long, so ordinary
 * integer arithmetic applies and the result is masked back to N bits when it
 * is stored; wider values support only construction, copying, bit/range
 * access and equality.
 */
#ifndef GDN_SHIM_AP_INT_H
#define GDN_SHIM_AP_INT_H

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <type_traits>

template <int W> struct ap_uint;

template <int W, bool Small = (W <= 64)> struct ap_uint_store;

template <int W> struct ap_uint_store<W, true> {
    uint64_t v[1];
    operator unsigned long long() const { return v[0]; }
};

template <int W> struct ap_uint_store<W, false> {
    uint64_t v[(W + 63) / 64];
};

template <int W> struct ap_range_ref;
template <int W> struct ap_bit_ref;

template <int W> struct ap_uint : ap_uint_store<W> {
    static constexpr int NW = (W + 63) / 64;
    static_assert(W > 0, "ap_uint width must be positive");

    void mask_top() {
        if (W % 64) this->v[NW - 1] &= (~0ull) >> (64 - (W % 64));
    }
    uint64_t word(int i) const { return i < NW ? this->v[i] : 0; }

    ap_uint() { std::memset(this->v, 0, sizeof(this->v)); }

    template <typename T, typename std::enable_if<std::is_integral<T>::value, int>::type = 0>
    ap_uint(T x) {
        const bool neg = std::is_signed<T>::value && x < 0;
        this->v[0] = (uint64_t)(long long)x;
        if (!std::is_signed<T>::value) this->v[0] = (uint64_t)(unsigned long long)x;
        for (int i = 1; i < NW; ++i) this->v[i] = neg ? ~0ull : 0ull;
        mask_top();
    }

    template <int W2> ap_uint(const ap_uint<W2> &o) {
        for (int i = 0; i < NW; ++i) this->v[i] = o.word(i);
        mask_top();
    }

    template <int W2> ap_uint(const ap_range_ref<W2> &r) : ap_uint(r.get()) {}
    template <int W2> ap_uint(const ap_bit_ref<W2> &b) : ap_uint((unsigned)(bool)b) {}

    bool get_bit(int i) const { return (this->v[i >> 6] >> (i & 63)) & 1u; }
    void set_bit(int i, bool b) {
        if (b) this->v[i >> 6] |= 1ull << (i & 63);
        else this->v[i >> 6] &= ~(1ull << (i & 63));
    }

    /* up to 64 bits starting at bit pos */
    uint64_t get_bits64(int pos, int nbits) const {
        const int w = pos >> 6, s = pos & 63;
        uint64_t val = this->v[w] >> s;
        if (s != 0 && s + nbits > 64 && w + 1 < NW) val |= this->v[w + 1] << (64 - s);
        return nbits >= 64 ? val : (val & ((1ull << nbits) - 1));
    }
    void set_bits64(int pos, int nbits, uint64_t value) {
        const int w = pos >> 6, s = pos & 63;
        const uint64_t mask = nbits >= 64 ? ~0ull : ((1ull << nbits) - 1);
        value &= mask;
        this->v[w] = (this->v[w] & ~(mask << s)) | (value << s);
        if (s != 0 && s + nbits > 64) {
            const int rem = s + nbits - 64;
            const uint64_t m2 = (1ull << rem) - 1;
            this->v[w + 1] = (this->v[w + 1] & ~m2) | (value >> (64 - s));
        }
    }

    /* bits [hi:lo] right-aligned */
    ap_uint<W> get_range(int hi, int lo) const {
        ap_uint<W> r;
        const int n = hi - lo + 1;
        for (int j = 0; j * 64 < n; ++j) {
            const int nb = (n - j * 64) < 64 ? (n - j * 64) : 64;
            r.v[j] = get_bits64(lo + j * 64, nb);
        }
        return r;
    }
    template <int W2> void set_range(int hi, int lo, const ap_uint<W2> &val) {
        const int n = hi - lo + 1;
        for (int j = 0; j * 64 < n; ++j) {
            const int nb = (n - j * 64) < 64 ? (n - j * 64) : 64;
            set_bits64(lo + j * 64, nb, val.word(j));
        }
    }

    ap_range_ref<W> range(int hi, int lo) { return ap_range_ref<W>(this, hi, lo); }
    ap_uint<W> range(int hi, int lo) const { return get_range(hi, lo); }
    ap_range_ref<W> operator()(int hi, int lo) { return range(hi, lo); }
    ap_uint<W> operator()(int hi, int lo) const { return get_range(hi, lo); }
    ap_bit_ref<W> operator[](int i) { return ap_bit_ref<W>(this, i); }
    bool operator[](int i) const { return get_bit(i); }

    unsigned long long to_uint64() const { return this->v[0]; }
    unsigned int to_uint() const { return (unsigned int)this->v[0]; }
    int to_int() const { return (int)this->v[0]; }
    long long to_int64() const { return (long long)this->v[0]; }
    int length() const { return W; }
};

template <int W> struct ap_range_ref {
    ap_uint<W> *p;
    int hi, lo;
    ap_range_ref(ap_uint<W> *p_, int hi_, int lo_) : p(p_), hi(hi_), lo(lo_) {}
    ap_range_ref(const ap_range_ref &) = default;

    ap_uint<W> get() const { return p->get_range(hi, lo); }
    operator unsigned long long() const { return get().word(0); }

    template <int W2> ap_range_ref &operator=(const ap_uint<W2> &val) {
        p->set_range(hi, lo, val);
        return *this;
    }
    ap_range_ref &operator=(unsigned long long val) {
        p->set_range(hi, lo, ap_uint<64>(val));
        return *this;
    }
    ap_range_ref &operator=(const ap_range_ref &o) {
        const ap_uint<W> val = o.get();
        p->set_range(hi, lo, val);
        return *this;
    }
    template <int W2> ap_range_ref &operator=(const ap_range_ref<W2> &o) {
        const ap_uint<W2> val = o.get();
        p->set_range(hi, lo, val);
        return *this;
    }
    unsigned long long to_uint64() const { return get().word(0); }
    unsigned int to_uint() const { return (unsigned int)get().word(0); }
};

template <int W> struct ap_bit_ref {
    ap_uint<W> *p;
    int i;
    ap_bit_ref(ap_uint<W> *p_, int i_) : p(p_), i(i_) {}
    ap_bit_ref(const ap_bit_ref &) = default;
    operator bool() const { return p->get_bit(i); }
    ap_bit_ref &operator=(bool b) {
        p->set_bit(i, b);
        return *this;
    }
    ap_bit_ref &operator=(const ap_bit_ref &o) {
        p->set_bit(i, (bool)o);
        return *this;
    }
};

/* Equality for wide values (narrow ones compare as integers). */
template <int W>
typename std::enable_if<(W > 64), bool>::type operator==(const ap_uint<W> &a, const ap_uint<W> &b) {
    return std::memcmp(a.v, b.v, sizeof(a.v)) == 0;
}
template <int W>
typename std::enable_if<(W > 64), bool>::type operator!=(const ap_uint<W> &a, const ap_uint<W> &b) {
    return !(a == b);
}

/* Signed variant: only declared so that headers naming it compile. */
template <int W> struct ap_int : ap_uint<W> {
    using ap_uint<W>::ap_uint;
};

#endif
