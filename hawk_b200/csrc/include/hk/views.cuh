// hawk_b200 device library: plane views.
//
// A plane is component-major structure-of-arrays with unit sample stride
// (hawk/emit/wrapper.py:1029-1066): component k of sample i of a Vector[W]
// plane sits at data[k * pitch + i], pitch = the mirror's compStride_; a
// Matrix[R, C] plane at data[(r * C + c) * pitch + i]; a Scalar plane at
// data[i].  Consecutive threads take consecutive samples, so every warp-wide
// access to one component is one contiguous 256-byte (f64) run.
//
// Reads of input planes go through the read-only data path and writes of
// output planes are streaming (evict-first) stores: every plane byte is
// touched exactly once per launch, so neither should displace reused lines
// (the lookup cells) from L1/L2.
//
// The body indexes a view with the sample index ``i`` its frame binds:
//   in[i]          -> the sample's value (Item for rank >= 1), eagerly loaded;
//   in[i].get()    -> the same value; scalar in[i].eval() -> the scalar;
//   out[i] = v     -> store;  out[i].get()/.eval() -> the value the plane held
//                     when the launch began (a Mutable read), out[i][k] /
//                     out[i](r, c) -> a reference to one component (a solve
//                     writes its result through it);
//   rows.data()[r] -> a row plane's element r (sample-sum rows).
//
// An input view may be staged (hk/stage.cuh): the frame copies each tile of
// its components into shared memory, `stage_off` bytes into the stage and
// `comp_bytes` apart, and the sample index carries the tile; a read then comes
// from shared memory, and from global memory when the index carries none.
#pragma once
#include "abi.cuh"
#include "item.cuh"

namespace hk {

struct SampleIndex {
    i64 g;                                // the global sample index
    const unsigned char* st = nullptr;    // the staged tile holding the sample, if any
    int local = 0;                        // the sample's place in that tile

    static HK_FI SampleIndex make(usize k) { return SampleIndex{static_cast<i64>(k)}; }
    HK_FI i64 global() const { return g; }
};

template <class T> HK_FI T ld_in(const T* p) {
#if defined(__CUDA_ARCH__)
    return __ldg(p);
#else
    return *p;
#endif
}

template <class T> HK_FI void st_out(T* p, T v) {
#if defined(__CUDA_ARCH__)
    __stcs(p, v);
#else
    *p = v;
#endif
}

// A rank-0 value read from a plane.
template <class T> struct Val {
    T x;
    HK_FI T eval() const { return x; }
    HK_FI T get() const { return x; }
    HK_FI T operator()() const { return x; }
    HK_FI operator T() const { return x; }
};

// ------------------------------------------------------------------ inputs

// per_sample and lookup roles: one element per sample (or a one-cell plane).
template <class T> struct ScalarIn {
    const T* p;
    u64 n;
    unsigned stage_off;
    HK_FI explicit ScalarIn(const abi::ScalarHandle& h, unsigned off = 0)
        : p(static_cast<const T*>(h.data)), n(h.samples), stage_off(off) {}
    HK_FI explicit ScalarIn(const abi::IntHandle& h, unsigned off = 0)
        : p(static_cast<const T*>(h.data)), n(h.samples), stage_off(off) {}
    HK_FI Val<T> operator[](const SampleIndex& i) const {
        if (i.st) return Val<T>{reinterpret_cast<const T*>(i.st + stage_off)[i.local]};
        return Val<T>{ld_in(p + i.g)};
    }
    HK_FI T cell() const { return ld_in(p); }
    HK_FI const T* data() const { return p; }
    HK_FI u64 samples() const { return n; }
};

// A sample of a vector or matrix input plane of more than kLazyElems elements,
// read element by element where it is used (a whole value that size would not
// fit a thread's registers).  Element (r, c) is component r * C + c.
constexpr int kLazyElems = 48;

template <class T, int R, int C> struct Slice;

template <class T, int R, int C> struct InRef {
    const T* q;
    u64 pitch;
    HK_FI T flat(int k) const { return ld_in(q + static_cast<u64>(k) * pitch); }
    HK_FI T at(int k) const { return flat(k); }
    HK_FI T at(int r, int c) const { return flat(r * C + c); }
    HK_FI T operator()(int k) const { return flat(k); }
    HK_FI T operator()(int r, int c) const { return flat(r * C + c); }
    HK_FI T operator[](int k) const { return flat(k); }
    static HK_HD constexpr int size() { return R * C; }
    // a read of the whole value stays this reference (element reads where used)
    HK_FI const InRef& get() const { return *this; }
    HK_FI const InRef& eval() const { return *this; }
};

template <class T, int N> struct VecIn {
    const T* p;
    u64 pitch;
    u64 n;
    unsigned stage_off, comp_bytes;
    HK_FI explicit VecIn(const abi::GRefMirror& m, unsigned off = 0, unsigned cb = 0)
        : p(reinterpret_cast<const T*>(m.data_)), pitch(m.compStride_), n(m.samples_), stage_off(off),
          comp_bytes(cb) {}
    HK_FI auto operator[](const SampleIndex& i) const {
        if constexpr (N > kLazyElems) {
            return InRef<T, N, 1>{p + i.g, pitch};
        } else {
        Item<T, N> r;
        if (i.st) {
#pragma unroll
            for (int k = 0; k < N; ++k)
                r.v[k] = reinterpret_cast<const T*>(i.st + stage_off + static_cast<unsigned>(k) * comp_bytes)[i.local];
            return r;
        }
#pragma unroll
        for (int k = 0; k < N; ++k) r.v[k] = ld_in(p + static_cast<u64>(k) * pitch + i.g);
        return r;
        }
    }
    HK_FI const T* data() const { return p; }
    HK_FI u64 samples() const { return n; }
};

template <class T, int R, int C> struct MatIn {
    const T* p;
    u64 pitch;
    u64 n;
    unsigned stage_off, comp_bytes;
    HK_FI explicit MatIn(const abi::GRefMirror& m, unsigned off = 0, unsigned cb = 0)
        : p(reinterpret_cast<const T*>(m.data_)), pitch(m.compStride_), n(m.samples_), stage_off(off),
          comp_bytes(cb) {}
    HK_FI auto operator[](const SampleIndex& i) const {
        if constexpr (R * C > kLazyElems) {
            return InRef<T, R, C>{p + i.g, pitch};
        } else {
        Item<T, R, C> a;
        if (i.st) {
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int c = 0; c < C; ++c)
                    a.m[r][c] = reinterpret_cast<const T*>(
                        i.st + stage_off + static_cast<unsigned>(r * C + c) * comp_bytes)[i.local];
            return a;
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int c = 0; c < C; ++c)
                a.m[r][c] = ld_in(p + static_cast<u64>(r * C + c) * pitch + i.g);
        return a;
        }
    }
    HK_FI const T* data() const { return p; }
    HK_FI u64 samples() const { return n; }
};

// ------------------------------------------------------------------ sinks

// A scalar Mutable / out plane, or a row plane of a sample sum.
template <class T> struct ScalarOut {
    T* p;
    u64 n;
    struct Ref {
        T* q;
        HK_FI void operator=(T v) const { st_out(q, v); }
        HK_FI void operator+=(T v) const { *q = *q + v; }
        HK_FI T eval() const { return *q; }
        HK_FI Val<T> get() const { return Val<T>{*q}; }   // a Mutable read: plane[i].get()()
        HK_FI operator T() const { return *q; }
    };
    HK_FI explicit ScalarOut(const abi::ScalarHandle& h) : p(static_cast<T*>(h.data)), n(h.samples) {}
    HK_FI explicit ScalarOut(const abi::IntHandle& h) : p(static_cast<T*>(h.data)), n(h.samples) {}
    HK_FI Ref operator[](const SampleIndex& i) const { return Ref{p + i.g}; }
    HK_FI T* data() const { return p; }
    HK_FI u64 samples() const { return n; }
};

// A finishing kernel's mask (the Terminated plane, one bool per sample): read
// at the top of the step and set by its finish epilogue in the same launch, so
// both go through the coherent path (never the read-only one).
struct MaskView {
    bool* p;
    u64 n;
    struct Ref {
        bool* q;
        HK_FI void operator=(bool v) const { *q = v; }
        HK_FI bool eval() const { return *q; }
        HK_FI operator bool() const { return *q; }
    };
    HK_FI explicit MaskView(const abi::ScalarHandle& h) : p(static_cast<bool*>(h.data)), n(h.samples) {}
    HK_FI Ref operator[](const SampleIndex& i) const { return Ref{p + i.g}; }
    HK_FI bool* data() const { return p; }
    HK_FI u64 samples() const { return n; }
};

template <class T, int N> struct VecOut {
    T* p;
    u64 pitch;
    u64 n;
    struct Ref {
        T* q;
        u64 pitch;
        HK_FI void operator=(const Item<T, N>& v) const {
#pragma unroll
            for (int k = 0; k < N; ++k) st_out(q + static_cast<u64>(k) * pitch, v.v[k]);
        }
        HK_FI void operator+=(const Item<T, N>& v) const {
#pragma unroll
            for (int k = 0; k < N; ++k) q[static_cast<u64>(k) * pitch] += v.v[k];
        }
        // a value that lives in a scratch slice: copied element by element
        template <int C2> HK_FI void operator=(const Slice<T, N, C2>& v) const {
#pragma unroll 16
            for (int k = 0; k < N; ++k) st_out(q + static_cast<u64>(k) * pitch, v.flat(k));
        }
        HK_FI T& operator[](int k) const { return q[static_cast<u64>(k) * pitch]; }
        HK_FI T& operator()(int k) const { return q[static_cast<u64>(k) * pitch]; }
        HK_FI T& flat(int k) const { return q[static_cast<u64>(k) * pitch]; }
        static HK_HD constexpr int size() { return N; }
        HK_FI T& at(int k) const { return q[static_cast<u64>(k) * pitch]; }
        HK_FI Item<T, N> get() const {
            Item<T, N> r;
#pragma unroll
            for (int k = 0; k < N; ++k) r.v[k] = q[static_cast<u64>(k) * pitch];
            return r;
        }
        HK_FI Item<T, N> eval() const { return get(); }
        HK_FI operator Item<T, N>() const { return get(); }
    };
    HK_FI explicit VecOut(const abi::GRefMirror& m)
        : p(reinterpret_cast<T*>(m.data_)), pitch(m.compStride_), n(m.samples_) {}
    HK_FI Ref operator[](const SampleIndex& i) const { return Ref{p + i.g, pitch}; }
    HK_FI T* data() const { return p; }
    HK_FI u64 samples() const { return n; }
};

template <class T, int R, int C> struct MatOut {
    T* p;
    u64 pitch;
    u64 n;
    struct Ref {
        T* q;
        u64 pitch;
        HK_FI void operator=(const Item<T, R, C>& a) const {
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int c = 0; c < C; ++c) st_out(q + static_cast<u64>(r * C + c) * pitch, a.m[r][c]);
        }
        // a value that lives in a scratch slice: copied element by element
        HK_FI void operator=(const Slice<T, R, C>& a) const {
#pragma unroll 16
            for (int k = 0; k < R * C; ++k) st_out(q + static_cast<u64>(k) * pitch, a.flat(k));
        }
        HK_FI T& operator()(int r, int c) const { return q[static_cast<u64>(r * C + c) * pitch]; }
        HK_FI T& at(int r, int c) const { return q[static_cast<u64>(r * C + c) * pitch]; }
        HK_FI T& flat(int k) const { return q[static_cast<u64>(k) * pitch]; }
        static HK_HD constexpr int size() { return R * C; }
        HK_FI Item<T, R, C> get() const {
            Item<T, R, C> a;
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int c = 0; c < C; ++c) a.m[r][c] = q[static_cast<u64>(r * C + c) * pitch];
            return a;
        }
        HK_FI Item<T, R, C> eval() const { return get(); }
        HK_FI operator Item<T, R, C>() const { return get(); }
    };
    HK_FI explicit MatOut(const abi::GRefMirror& m)
        : p(reinterpret_cast<T*>(m.data_)), pitch(m.compStride_), n(m.samples_) {}
    HK_FI Ref operator[](const SampleIndex& i) const { return Ref{p + i.g, pitch}; }
    HK_FI T* data() const { return p; }
    HK_FI u64 samples() const { return n; }
};


// A vector or matrix a team stage left row-major in the lane's slice of a
// scratch plane (the reader stage's view of it): element k is p[k].
template <class T, int R, int C = 1> struct Slice {
    const T* p;
    HK_FI T flat(int k) const { return p[k]; }
    HK_FI T at(int k) const { return p[k]; }
    HK_FI T at(int r, int c) const { return p[r * C + c]; }
    HK_FI T operator()(int k) const { return p[k]; }
    HK_FI T operator()(int r, int c) const { return p[r * C + c]; }
    HK_FI T operator[](int k) const { return p[k]; }
    HK_FI const T* data() const { return p; }
    static HK_HD constexpr int size() { return R * C; }
    // the whole value, for an operation on all of it (held in registers or
    // local memory: what the one-thread form of the same value costs)
    HK_FI auto expr() const {
        if constexpr (C == 1) {
            Item<T, R> v;
            for (int k = 0; k < R; ++k) v.v[k] = p[k];
            return v;
        } else {
            Item<T, R, C> v;
            for (int k = 0; k < R * C; ++k) v.data()[k] = p[k];
            return v;
        }
    }
    HK_FI auto get() const { return expr(); }
    HK_FI auto eval() const { return expr(); }
};

namespace rt {
namespace detail {
template <class S> HK_FI auto flat_of(const S& s, int k) -> decltype(s.flat(k)) { return s.flat(k); }
template <class T, int... D> HK_FI T flat_of(const Item<T, D...>& s, int k) { return s.data()[k]; }
}  // namespace detail

// dst = src element by element in a rolled loop: a value of hundreds or
// thousands of elements (a factor read back from a team stage) is copied
// straight from where it lives into the output plane, never held whole.
template <class Dst, class Src> HK_FI void store(const Dst& dst, const Src& src) {
#pragma unroll 16
    for (int k = 0; k < Dst::size(); ++k) dst.flat(k) = detail::flat_of(src, k);
}
}  // namespace rt

}  // namespace hk
