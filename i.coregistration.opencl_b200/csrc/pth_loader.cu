// SPDX-License-Identifier: Unlicense
//
// Weight-file reader behind the reference's pth_loader.h API
// (pth_loader.c:1148-1403 of the reference), for the three formats the
// reference reads:
//
//   - torch.save zip archives (PyTorch >= 1.6): data.pkl holds the pickled
//     object, data/<key> each storage as a stored (uncompressed) entry;
//     zip64 records are followed (pth_loader.c:66-178);
//   - the legacy torch.save stream (torch < 1.6, or
//     _use_new_zipfile_serialization=False): five pickles, then every
//     storage as an int64 element count and its raw elements
//     (pth_loader.c:870-930);
//   - safetensors: an 8-byte header length, a JSON header, the data
//     (pth_loader.c:1014-1146).
//
// The pickled object is evaluated by a small unpickler that knows what a
// state_dict pickles to: dicts / OrderedDicts of tensors rebuilt from
// persistent storage references (torch._utils._rebuild_tensor_v2 and
// friends). Other callables become opaque objects, and an unknown opcode
// is an error. The state_dict is the pickled dict itself when it holds a
// tensor, else its "model" or "state_dict" entry, else its only entry that
// is a dict of tensors (DISK's "extractor"), as in pth_loader.c:706-740.
// Only float32 / float16 / bfloat16 tensors are indexed; integer and
// boolean ones (BatchNorm's num_batches_tracked) are left out.
//
// Every failure goes through coreg::fail: fatal in the reference's mode,
// recorded (pth_open leaves an empty pth_file) in the recording mode.

#include <fcntl.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <deque>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "pth_loader.h"

using coreg::fail;
using coreg::pending;

namespace {

// ------------------------------------------------------------- plumbing

// Parse errors are thrown as Bad and turned into one fail() by pth_open.
struct Bad {
    std::string msg;
};

[[noreturn]] void bad(const char *fmt, ...) __attribute__((format(printf, 1, 2)));

void bad(const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    throw Bad{buf};
}

uint64_t le(const unsigned char *p, int n)
{
    uint64_t v = 0;
    for (int i = n - 1; i >= 0; i--)
        v = v << 8 | p[i];
    return v;
}

size_t dtype_bytes(enum pth_dtype d) { return d == PTH_F32 ? 4 : 2; }

// The whole file, mapped read-only for parsing.
struct Mapped {
    const unsigned char *p = nullptr;
    size_t n = 0;

    Mapped(const Mapped &) = delete;
    Mapped &operator=(const Mapped &) = delete;
    Mapped(FILE *fp, const char *path)
    {
        struct stat st;
        if (fstat(fileno(fp), &st) != 0)
            bad("Unable to stat checkpoint <%s>", path);
        n = (size_t)st.st_size;
        if (n == 0)
            return;
        void *m = mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fileno(fp), 0);
        if (m == MAP_FAILED)
            bad("Unable to map checkpoint <%s>", path);
        p = (const unsigned char *)m;
    }
    ~Mapped()
    {
        if (p)
            munmap((void *)p, n);
    }
    // Bytes [off, off + len) of the file, or an error naming what.
    const unsigned char *at(uint64_t off, uint64_t len, const char *what) const
    {
        if (off > n || len > n - off)
            bad("Truncated checkpoint: %s lies past the end of the file", what);
        return p + off;
    }
};

// ------------------------------------------------------------------ zip

struct ZipEntry {
    std::string name;
    int method;
    uint64_t size, local;
};

// The central directory, found from the end-of-central-directory record
// (searched backwards over the 64 KiB comment window), through the zip64
// locator and record when the classic fields overflow.
std::vector<ZipEntry> zip_entries(const Mapped &f, const char *path)
{
    const size_t tail = f.n < 65557 ? f.n : 65557;
    long eocd = -1;
    for (long i = (long)f.n - 22; i >= (long)(f.n - tail); i--)
        if (le(f.p + i, 4) == 0x06054b50u) {
            eocd = i;
            break;
        }
    if (eocd < 0)
        bad("<%s> is not a zip archive (PyTorch >= 1.6 checkpoint format "
            "expected)",
            path);
    const unsigned char *e = f.p + eocd;
    uint64_t count = le(e + 10, 2), dir_bytes = le(e + 12, 4), dir_off = le(e + 16, 4);
    if (count == 0xffff || dir_bytes == 0xffffffffu || dir_off == 0xffffffffu) {
        if (eocd < 20 || le(e - 20, 4) != 0x07064b50u)
            bad("Corrupt zip64 directory in <%s>", path);
        const unsigned char *r = f.at(le(e - 20 + 8, 8), 56, "the zip64 end record");
        if (le(r, 4) != 0x06064b50u)
            bad("Corrupt zip64 end record in <%s>", path);
        count = le(r + 32, 8);
        dir_bytes = le(r + 40, 8);
        dir_off = le(r + 48, 8);
    }
    const unsigned char *d = f.at(dir_off, dir_bytes, "the zip central directory");
    const unsigned char *end = d + dir_bytes;
    std::vector<ZipEntry> out;
    out.reserve(count);
    for (uint64_t k = 0; k < count; k++) {
        if (end - d < 46 || le(d, 4) != 0x02014b50u)
            bad("Corrupt zip central directory in <%s>", path);
        const unsigned nlen = le(d + 28, 2), xlen = le(d + 30, 2), clen = le(d + 32, 2);
        if ((size_t)(end - d) < 46u + nlen + xlen + clen)
            bad("Corrupt zip central directory in <%s>", path);
        ZipEntry z;
        z.method = (int)le(d + 10, 2);
        const uint64_t csize = le(d + 20, 4);
        z.size = le(d + 24, 4);
        z.local = le(d + 42, 4);
        z.name.assign((const char *)d + 46, nlen);
        // The zip64 extra field holds, in this order, whichever of the
        // uncompressed size, compressed size and local offset overflowed.
        for (const unsigned char *x = d + 46 + nlen, *xe = x + xlen; xe - x >= 4;) {
            const unsigned id = le(x, 2), len = le(x + 2, 2);
            const unsigned char *v = x + 4, *ve = v + len;
            if (ve > xe)
                break;
            if (id == 0x0001) {
                if (z.size == 0xffffffffu && ve - v >= 8) {
                    z.size = le(v, 8);
                    v += 8;
                }
                if (csize == 0xffffffffu && ve - v >= 8)
                    v += 8;
                if (z.local == 0xffffffffu && ve - v >= 8)
                    z.local = le(v, 8);
            }
            x = ve;
        }
        out.push_back(std::move(z));
        d += 46 + nlen + xlen + clen;
    }
    return out;
}

// File offset of an entry's bytes, after its local header.
uint64_t zip_payload(const Mapped &f, const ZipEntry &z, const char *path)
{
    if (z.method != 0)
        bad("Zip entry <%s> in <%s> is compressed; only stored entries (as "
            "written by torch.save) are supported",
            z.name.c_str(), path);
    const unsigned char *h = f.at(z.local, 30, "a zip local header");
    if (le(h, 4) != 0x04034b50u)
        bad("Corrupt local header for <%s> in <%s>", z.name.c_str(), path);
    const uint64_t off = z.local + 30 + le(h + 26, 2) + le(h + 28, 2);
    f.at(off, z.size, "a zip entry");
    return off;
}

// --------------------------------------------------------------- pickle

enum class Kind : uint8_t {
    None,
    Bool,
    Int,
    Float,
    Str,
    Bytes,
    Tuple,
    List,
    Dict,
    Global,
    Storage,
    Tensor,
    Opaque
};

struct Obj {
    Kind kind;
    long ival = 0;
    double fval = 0;
    std::string text;  // Str / Bytes payload; Global module; Storage key.
    std::string name;  // Global qualified name.
    std::vector<Obj *> items;  // Tuple / List; Dict as key, value, key, ...
    // Storage: element type and size in bytes.
    enum pth_dtype dtype = PTH_OTHER;
    int elsize = 0;
    // Tensor: a view of a storage.
    const Obj *storage = nullptr;
    long offset = 0;
    int ndim = 0;
    long shape[PTH_MAX_DIMS] = {}, stride[PTH_MAX_DIMS] = {};

    explicit Obj(Kind k) : kind(k) {}
    bool is(const char *mod, const char *qual) const
    {
        return kind == Kind::Global && text == mod && name == qual;
    }
};

// The storage types torch pickles (torch.<Name>Storage) and their element
// sizes; the floating ones are the types a state_dict is indexed by.
struct StorageType {
    const char *name;
    enum pth_dtype dtype;
    int elsize;
};
const StorageType kStorageTypes[] = {
    {"FloatStorage", PTH_F32, 4},   {"HalfStorage", PTH_F16, 2},
    {"BFloat16Storage", PTH_BF16, 2}, {"DoubleStorage", PTH_OTHER, 8},
    {"LongStorage", PTH_OTHER, 8},  {"IntStorage", PTH_OTHER, 4},
    {"ShortStorage", PTH_OTHER, 2}, {"CharStorage", PTH_OTHER, 1},
    {"ByteStorage", PTH_OTHER, 1},  {"BoolStorage", PTH_OTHER, 1},
    {"UntypedStorage", PTH_OTHER, 1},
};

class Unpickler {
  public:
    Unpickler(const unsigned char *p, const unsigned char *end) : p_(p), end_(end) {}

    // Evaluate one pickle, up to its STOP; returns the object it built.
    Obj *load()
    {
        stack_.clear();
        marks_.clear();
        memo_.clear();
        for (;;) {
            const long at = pos_;
            const unsigned char op = *take(1);
            if (op == '.') {
                if (stack_.empty())
                    bad("Empty pickle stack at STOP");
                return stack_.back();
            }
            step(op, at);
        }
    }
    size_t consumed() const { return (size_t)pos_; }
    const std::deque<Obj> &objects() const { return arena_; }

  private:
    const unsigned char *p_, *end_;
    long pos_ = 0;
    std::deque<Obj> arena_;  // Stable addresses; freed with the unpickler.
    std::vector<Obj *> stack_;
    std::vector<size_t> marks_;
    std::unordered_map<uint64_t, Obj *> memo_;

    const unsigned char *take(size_t n)
    {
        if ((size_t)(end_ - p_) < (size_t)pos_ || (size_t)(end_ - p_) - (size_t)pos_ < n)
            bad("Truncated pickle");
        const unsigned char *r = p_ + pos_;
        pos_ += (long)n;
        return r;
    }
    std::string line()
    {
        const unsigned char *s = p_ + pos_;
        const void *nl = memchr(s, '\n', (size_t)(end_ - s));
        if (!nl)
            bad("Truncated pickle");
        const size_t n = (const unsigned char *)nl - s;
        pos_ += (long)n + 1;
        return std::string((const char *)s, n);
    }
    Obj *make(Kind k)
    {
        arena_.emplace_back(k);
        return &arena_.back();
    }
    Obj *make_int(long v)
    {
        Obj *o = make(Kind::Int);
        o->ival = v;
        return o;
    }
    Obj *make_text(Kind k, const unsigned char *s, size_t n)
    {
        Obj *o = make(k);
        o->text.assign((const char *)s, n);
        return o;
    }
    void push(Obj *o) { stack_.push_back(o); }
    Obj *pop()
    {
        if (stack_.empty() || (!marks_.empty() && stack_.size() <= marks_.back()))
            bad("Pickle stack underflow");
        Obj *o = stack_.back();
        stack_.pop_back();
        return o;
    }
    Obj *top()
    {
        if (stack_.empty())
            bad("Pickle stack underflow");
        return stack_.back();
    }
    // The objects pushed since the last MARK, which is dropped.
    std::vector<Obj *> pop_mark()
    {
        if (marks_.empty())
            bad("Pickle MARK missing");
        const size_t m = marks_.back();
        marks_.pop_back();
        std::vector<Obj *> v(stack_.begin() + m, stack_.end());
        stack_.resize(m);
        return v;
    }
    Obj *tuple(std::vector<Obj *> items)
    {
        Obj *t = make(Kind::Tuple);
        t->items = std::move(items);
        return t;
    }
    void memo_put(uint64_t idx) { memo_[idx] = top(); }
    Obj *memo_get(uint64_t idx)
    {
        auto it = memo_.find(idx);
        if (it == memo_.end())
            bad("Pickle memo entry %lu missing", (unsigned long)idx);
        return it->second;
    }
    static long as_int(const Obj *o)
    {
        if (o->kind != Kind::Int && o->kind != Kind::Bool)
            bad("Integer expected in a tensor's arguments");
        return o->ival;
    }
    void add_items(Obj *target, const std::vector<Obj *> &v)
    {
        if (target->kind == Kind::Dict || target->kind == Kind::List)
            target->items.insert(target->items.end(), v.begin(), v.end());
        // Items of an opaque object do not matter for a state_dict.
    }
    Obj *global(std::string mod, std::string qual)
    {
        Obj *g = make(Kind::Global);
        g->text = std::move(mod);
        g->name = std::move(qual);
        return g;
    }

    // BINPERSID: a storage reference of torch.save,
    // ("storage", torch.<Type>Storage, key, location, numel[, view]).
    Obj *persistent(const Obj *pid)
    {
        if (pid->kind != Kind::Tuple || pid->items.size() < 5 ||
            pid->items[0]->kind != Kind::Str || pid->items[0]->text != "storage" ||
            pid->items[1]->kind != Kind::Global || pid->items[2]->kind != Kind::Str)
            bad("Unsupported persistent id in checkpoint");
        const Obj *type = pid->items[1];
        Obj *s = make(Kind::Storage);
        for (const StorageType &t : kStorageTypes)
            if (type->text == "torch" && type->name == t.name) {
                s->dtype = t.dtype;
                s->elsize = t.elsize;
            }
        if (!s->elsize)
            bad("Unsupported tensor storage type <%s.%s> in checkpoint", type->text.c_str(),
                type->name.c_str());
        s->text = pid->items[2]->text;
        return s;
    }

    // REDUCE: the callables a state_dict is made of.
    Obj *call(const Obj *fn, const Obj *args)
    {
        if (args->kind != Kind::Tuple)
            bad("Pickle REDUCE without an argument tuple");
        const std::vector<Obj *> &a = args->items;
        const bool v3 = fn->is("torch._utils", "_rebuild_tensor_v3");
        if (fn->is("torch._utils", "_rebuild_tensor_v2") ||
            fn->is("torch._utils", "_rebuild_tensor") || v3) {
            // (storage, storage_offset, size, stride, ...)
            if (a.size() < 4 || a[0]->kind != Kind::Storage || a[2]->kind != Kind::Tuple ||
                a[3]->kind != Kind::Tuple)
                bad("Unexpected tensor rebuild arguments");
            const Obj *size = a[2], *stride = a[3];
            if (size->items.size() > PTH_MAX_DIMS || size->items.size() != stride->items.size())
                bad("Unsupported tensor rank %zu", size->items.size());
            Obj *t = make(Kind::Tensor);
            t->storage = a[0];
            t->offset = as_int(a[1]);
            t->ndim = (int)size->items.size();
            for (int d = 0; d < t->ndim; d++) {
                t->shape[d] = as_int(size->items[d]);
                t->stride[d] = as_int(stride->items[d]);
            }
            // v3 carries its dtype apart from an untyped storage; only
            // dtypes outside the float32 / float16 / bfloat16 set use it.
            if (v3) {
                Obj *s = make(Kind::Storage);
                *s = *a[0];
                s->dtype = PTH_OTHER;
                t->storage = s;
            }
            return t;
        }
        if (fn->is("torch._utils", "_rebuild_parameter") ||
            fn->is("torch._utils", "_rebuild_parameter_with_state")) {
            if (a.empty() || a[0]->kind != Kind::Tensor)
                bad("Unexpected parameter rebuild arguments");
            return a[0];
        }
        // A tensor subclass, or a tensor with Python attributes (DINOv2's
        // checkpoint): (rebuild function, type, its arguments, state); the
        // type and the state leave the data alone.
        if (fn->is("torch._tensor", "_rebuild_from_type_v2")) {
            if (a.size() < 3 || a[0]->kind != Kind::Global || a[2]->kind != Kind::Tuple)
                bad("Unexpected tensor subclass rebuild arguments");
            return call(a[0], a[2]);
        }
        if (fn->is("collections", "OrderedDict"))
            return make(Kind::Dict);
        return make(Kind::Opaque);
    }

    void step(unsigned char op, long at)
    {
        switch (op) {
        case 0x80:  // PROTO
            take(1);
            break;
        case 0x95:  // FRAME: frames only group the opcodes that follow.
            take(8);
            break;
        case '(':  // MARK
            marks_.push_back(stack_.size());
            break;
        case '}':  // EMPTY_DICT
            push(make(Kind::Dict));
            break;
        case ']':  // EMPTY_LIST
            push(make(Kind::List));
            break;
        case ')':  // EMPTY_TUPLE
            push(tuple({}));
            break;
        case 0x8f:  // EMPTY_SET
            push(make(Kind::Opaque));
            break;
        case 'N':
            push(make(Kind::None));
            break;
        case 0x88:  // NEWTRUE
        case 0x89: {  // NEWFALSE
            Obj *b = make(Kind::Bool);
            b->ival = op == 0x88;
            push(b);
            break;
        }
        case 'J':  // BININT
            push(make_int((int32_t)le(take(4), 4)));
            break;
        case 'K':  // BININT1
            push(make_int((long)*take(1)));
            break;
        case 'M':  // BININT2
            push(make_int((long)le(take(2), 2)));
            break;
        case 0x8a:    // LONG1
        case 0x8b: {  // LONG4
            const size_t n = op == 0x8a ? *take(1) : (size_t)le(take(4), 4);
            const unsigned char *b = take(n);
            if (n > 8) {
                // Wider than a long: the legacy stream's magic number,
                // which no state_dict entry needs.
                push(make(Kind::Opaque));
                break;
            }
            uint64_t v = n ? le(b, (int)n) : 0;
            if (n && n < 8 && (b[n - 1] & 0x80))
                v |= ~(uint64_t)0 << (8 * n);  // Two's complement sign.
            push(make_int((long)v));
            break;
        }
        case 'I':    // INT (text; 00 / 01 are the booleans of protocol 0)
        case 'L': {  // LONG (text)
            std::string s = line();
            if (op == 'I' && (s == "00" || s == "01")) {
                Obj *b = make(Kind::Bool);
                b->ival = s == "01";
                push(b);
            }
            else
                push(make_int(strtol(s.c_str(), nullptr, 10)));
            break;
        }
        case 'G': {  // BINFLOAT, big-endian
            const unsigned char *b = take(8);
            uint64_t u = 0;
            for (int i = 0; i < 8; i++)
                u = u << 8 | b[i];
            Obj *f = make(Kind::Float);
            memcpy(&f->fval, &u, 8);
            push(f);
            break;
        }
        case 'X':  // BINUNICODE
        case 'T': {  // BINSTRING
            const size_t n = (size_t)le(take(4), 4);
            push(make_text(Kind::Str, take(n), n));
            break;
        }
        case 0x8c:  // SHORT_BINUNICODE
        case 'U': {  // SHORT_BINSTRING
            const size_t n = *take(1);
            push(make_text(Kind::Str, take(n), n));
            break;
        }
        case 0x8d: {  // BINUNICODE8
            const size_t n = (size_t)le(take(8), 8);
            push(make_text(Kind::Str, take(n), n));
            break;
        }
        case 'B':  // BINBYTES
        case 'C':  // SHORT_BINBYTES
        case 0x8e: {  // BINBYTES8
            const int w = op == 'C' ? 1 : op == 'B' ? 4 : 8;
            const size_t n = (size_t)le(take(w), w);
            push(make_text(Kind::Bytes, take(n), n));
            break;
        }
        case 'c': {  // GLOBAL: module and name, one text line each
            std::string mod = line();
            std::string qual = line();
            push(global(std::move(mod), std::move(qual)));
            break;
        }
        case 0x93: {  // STACK_GLOBAL
            Obj *qual = pop(), *mod = pop();
            if (qual->kind != Kind::Str || mod->kind != Kind::Str)
                bad("Pickle STACK_GLOBAL without names");
            push(global(mod->text, qual->text));
            break;
        }
        case 'q':  // BINPUT
            memo_put(*take(1));
            break;
        case 'r':  // LONG_BINPUT
            memo_put(le(take(4), 4));
            break;
        case 0x94:  // MEMOIZE
            memo_put(memo_.size());
            break;
        case 'p':  // PUT (text)
            memo_put(strtoul(line().c_str(), nullptr, 10));
            break;
        case 'h':  // BINGET
            push(memo_get(*take(1)));
            break;
        case 'j':  // LONG_BINGET
            push(memo_get(le(take(4), 4)));
            break;
        case 'g':  // GET (text)
            push(memo_get(strtoul(line().c_str(), nullptr, 10)));
            break;
        case '0':  // POP
            if (!marks_.empty() && marks_.back() == stack_.size())
                marks_.pop_back();
            else
                pop();
            break;
        case '1':  // POP_MARK
            pop_mark();
            break;
        case '2':  // DUP
            push(top());
            break;
        case 't':  // TUPLE
            push(tuple(pop_mark()));
            break;
        case 0x85:  // TUPLE1
        case 0x86:  // TUPLE2
        case 0x87: {  // TUPLE3
            std::vector<Obj *> v(op - 0x84);
            for (size_t i = v.size(); i-- > 0;)
                v[i] = pop();
            push(tuple(std::move(v)));
            break;
        }
        case 'l': {  // LIST
            Obj *l = make(Kind::List);
            l->items = pop_mark();
            push(l);
            break;
        }
        case 'd': {  // DICT
            Obj *d = make(Kind::Dict);
            d->items = pop_mark();
            if (d->items.size() % 2)
                bad("Pickle DICT with an odd number of items");
            push(d);
            break;
        }
        case 'Q': {  // BINPERSID
            Obj *pid = pop();
            push(persistent(pid));
            break;
        }
        case 'R': {  // REDUCE
            Obj *args = pop(), *fn = pop();
            push(call(fn, args));
            break;
        }
        case 0x81: {  // NEWOBJ: cls.__new__(cls, *args)
            pop();
            Obj *cls = pop();
            push(make(cls->is("collections", "OrderedDict") ? Kind::Dict : Kind::Opaque));
            break;
        }
        case 0x92: {  // NEWOBJ_EX: cls.__new__(cls, *args, **kwargs)
            pop();
            pop();
            Obj *cls = pop();
            push(make(cls->is("collections", "OrderedDict") ? Kind::Dict : Kind::Opaque));
            break;
        }
        case 'b':  // BUILD: the state (OrderedDict's _metadata and the like)
            pop();  // does not change a state_dict's entries.
            break;
        case 's': {  // SETITEM
            Obj *v = pop(), *k = pop();
            add_items(top(), {k, v});
            break;
        }
        case 'u': {  // SETITEMS
            std::vector<Obj *> kv = pop_mark();
            if (kv.size() % 2)
                bad("Pickle SETITEMS with an odd number of items");
            add_items(top(), kv);
            break;
        }
        case 'a': {  // APPEND
            Obj *v = pop();
            add_items(top(), {v});
            break;
        }
        case 'e':  // APPENDS
        case 0x90: {  // ADDITEMS
            std::vector<Obj *> v = pop_mark();
            add_items(top(), v);
            break;
        }
        case 0x91:  // FROZENSET
            pop_mark();
            push(make(Kind::Opaque));
            break;
        default:
            bad("Unsupported pickle opcode 0x%02x at offset %ld", op, at);
        }
    }
};

bool has_tensors(const Obj *d)
{
    for (size_t k = 1; k < d->items.size(); k += 2)
        if (d->items[k]->kind == Kind::Tensor)
            return true;
    return false;
}

// The state_dict inside the pickled object (pth_loader.c:706-740).
const Obj *find_state_dict(const Obj *root)
{
    if (root->kind != Kind::Dict)
        return nullptr;
    if (has_tensors(root))
        return root;
    const Obj *only = nullptr;
    int n = 0;
    for (size_t k = 0; k + 1 < root->items.size(); k += 2) {
        const Obj *key = root->items[k], *val = root->items[k + 1];
        if (key->kind != Kind::Str || val->kind != Kind::Dict || !has_tensors(val))
            continue;
        if (key->text == "model" || key->text == "state_dict")
            return val;
        only = val;
        n++;
    }
    return n == 1 ? only : nullptr;
}

// Storage key -> (file offset, bytes).
struct StorageRef {
    uint64_t offset, bytes;
};
using StorageIndex = std::unordered_map<std::string, StorageRef>;

// torch.save zip archive: the archive's folder is named after the saved
// file, so data.pkl is found by its suffix and the storages under the
// same folder's data/.
const Obj *open_zip(const Mapped &f, const char *path, Unpickler *&up, StorageIndex &ix)
{
    std::vector<ZipEntry> zs = zip_entries(f, path);
    const ZipEntry *pkl = nullptr;
    for (const ZipEntry &z : zs) {
        const size_t n = z.name.size();
        if (n >= 8 && z.name.compare(n - 8, 8, "data.pkl") == 0 &&
            (n == 8 || z.name[n - 9] == '/')) {
            pkl = &z;
            break;
        }
    }
    if (!pkl)
        bad("No data.pkl in <%s>: not a PyTorch checkpoint", path);
    const std::string data = pkl->name.substr(0, pkl->name.size() - 8) + "data/";
    const uint64_t off = zip_payload(f, *pkl, path);
    up = new Unpickler(f.p + off, f.p + off + pkl->size);
    const Obj *sd = find_state_dict(up->load());
    for (const ZipEntry &z : zs)
        if (z.name.size() > data.size() && z.name.compare(0, data.size(), data) == 0)
            ix[z.name.substr(data.size())] = {zip_payload(f, z, path), z.size};
    return sd;
}

// Legacy stream: magic number, protocol version (1001), system
// information, the object, the list of storage keys; then each listed
// storage as a little-endian int64 element count and its elements, whose
// size comes from the storage type the object named.
const Obj *open_legacy(const Mapped &f, const char *path, Unpickler *&up, StorageIndex &ix)
{
    if (f.n < 2 || f.p[0] != 0x80)
        bad("<%s> is neither a zip archive nor a legacy pickle: not a PyTorch checkpoint",
            path);
    up = new Unpickler(f.p, f.p + f.n);
    up->load();  // Magic number.
    const Obj *proto = up->load();
    if (proto->kind != Kind::Int || proto->ival != 1001)
        bad("<%s> is neither a zip archive nor a legacy PyTorch checkpoint", path);
    up->load();  // System information.
    const Obj *sd = find_state_dict(up->load());
    const Obj *keys = up->load();
    if (keys->kind != Kind::List)
        bad("<%s>: no storage key list after the object", path);
    std::unordered_map<std::string, int> elsize;
    for (const Obj &o : up->objects())
        if (o.kind == Kind::Storage)
            elsize.emplace(o.text, o.elsize);
    uint64_t off = up->consumed();
    for (const Obj *k : keys->items) {
        if (k->kind != Kind::Str)
            bad("<%s>: invalid storage key", path);
        auto es = elsize.find(k->text);
        if (es == elsize.end())
            bad("<%s>: storage <%s> is not used by any tensor", path, k->text.c_str());
        const uint64_t numel = le(f.at(off, 8, "a storage size"), 8);
        off += 8;
        if (numel > f.n / (uint64_t)es->second)
            bad("Truncated checkpoint <%s>", path);
        const uint64_t bytes = numel * (uint64_t)es->second;
        f.at(off, bytes, "a storage");
        ix[k->text] = {off, bytes};
        off += bytes;
    }
    return sd;
}

// The state_dict's float tensors, in the pickled order, checked against
// their storages (every strided element inside it).
std::vector<struct pth_tensor> index_state_dict(const Obj *sd, const StorageIndex &ix,
                                                const char *path)
{
    std::vector<struct pth_tensor> ts;
    try {
    for (size_t k = 1; k < sd->items.size(); k += 2) {
        const Obj *key = sd->items[k - 1], *tv = sd->items[k];
        if (tv->kind != Kind::Tensor || key->kind != Kind::Str ||
            tv->storage->dtype == PTH_OTHER)
            continue;
        struct pth_tensor t;
        memset(&t, 0, sizeof(t));
        t.ndim = tv->ndim;
        t.storage_offset = tv->offset;
        t.dtype = tv->storage->dtype;
        long last = tv->offset;
        for (int d = 0; d < tv->ndim; d++) {
            t.shape[d] = tv->shape[d];
            t.stride[d] = tv->stride[d];
            if (t.shape[d] <= 0)
                bad("Empty tensor <%s> in checkpoint", key->text.c_str());
            if (t.stride[d] < 0)
                bad("Tensor <%s> has a negative stride", key->text.c_str());
            last += (t.shape[d] - 1) * t.stride[d];
        }
        auto s = ix.find(tv->storage->text);
        if (s == ix.end())
            bad("Storage <%s> of tensor <%s> missing in <%s>", tv->storage->text.c_str(),
                key->text.c_str(), path);
        t.data_offset = (off_t)s->second.offset;
        t.storage_bytes = (size_t)s->second.bytes;
        if (t.storage_offset < 0 ||
            (uint64_t)(last + 1) * dtype_bytes(t.dtype) > t.storage_bytes)
            bad("Tensor <%s> exceeds its storage in <%s>", key->text.c_str(), path);
        t.name = strdup(key->text.c_str());
        ts.push_back(t);
    }
    }
    catch (...) {
        for (auto &t : ts)
            free(t.name);
        throw;
    }
    return ts;
}

// ----------------------------------------------------------- safetensors

// Minimal JSON reader for the safetensors header: objects, arrays,
// strings, integers; other values are skipped.
struct Json {
    const char *s, *e;

    void ws()
    {
        while (s < e && (*s == ' ' || *s == '\n' || *s == '\r' || *s == '\t'))
            s++;
    }
    bool eat(char c)
    {
        ws();
        if (s < e && *s == c) {
            s++;
            return true;
        }
        return false;
    }
    void expect(char c)
    {
        if (!eat(c))
            bad("malformed safetensors header: '%c' expected", c);
    }
    std::string str()
    {
        ws();
        if (s >= e || *s != '"')
            bad("malformed safetensors header: string expected");
        std::string out;
        for (s++; s < e && *s != '"'; s++) {
            if (*s == '\\' && s + 1 < e) {
                s++;
                out += *s == 'n' ? '\n' : *s == 't' ? '\t' : *s;
            }
            else
                out += *s;
        }
        if (s >= e)
            bad("malformed safetensors header: unterminated string");
        s++;
        return out;
    }
    long num()
    {
        ws();
        char *end;
        const long v = strtol(s, &end, 10);
        if (end == s)
            bad("malformed safetensors header: integer expected");
        s = end;
        return v;
    }
    void skip()
    {
        ws();
        if (s >= e)
            bad("malformed safetensors header");
        if (*s == '"')
            str();
        else if (*s == '{' || *s == '[') {
            const char close = *s == '{' ? '}' : ']';
            s++;
            if (eat(close))
                return;
            do {
                if (close == '}') {
                    str();
                    expect(':');
                }
                skip();
            } while (eat(','));
            expect(close);
        }
        else
            while (s < e && *s != ',' && *s != '}' && *s != ']')
                s++;
    }
};

// A safetensors file if its first 9 bytes say so (a header length that
// fits the file, then '{'); tensors of other dtypes than F32, F16 and
// BF16 are left out.
bool is_safetensors(const Mapped &f)
{
    if (f.n < 9 || f.p[8] != '{')
        return false;
    const uint64_t h = le(f.p, 8);
    return h >= 2 && h <= f.n - 8;
}

std::vector<struct pth_tensor> open_safetensors(const Mapped &f, const char *path)
{
    const uint64_t hlen = le(f.p, 8);
    Json j{(const char *)f.p + 8, (const char *)f.p + 8 + hlen};
    std::vector<struct pth_tensor> ts;
    try {
        j.expect('{');
        if (!j.eat('}'))
            do {
                const std::string name = j.str();
                j.expect(':');
                if (name == "__metadata__") {
                    j.skip();
                    continue;
                }
                std::string dtype;
                std::vector<long> shape;
                long off0 = -1, off1 = -1;
                j.expect('{');
                if (!j.eat('}'))
                    do {
                        const std::string key = j.str();
                        j.expect(':');
                        if (key == "dtype")
                            dtype = j.str();
                        else if (key == "shape") {
                            j.expect('[');
                            if (!j.eat(']')) {
                                do
                                    shape.push_back(j.num());
                                while (j.eat(','));
                                j.expect(']');
                            }
                        }
                        else if (key == "data_offsets") {
                            j.expect('[');
                            off0 = j.num();
                            j.expect(',');
                            off1 = j.num();
                            j.expect(']');
                        }
                        else
                            j.skip();
                    } while (j.eat(','));
                    j.expect('}');
                const enum pth_dtype dt = dtype == "F32"    ? PTH_F32
                                          : dtype == "F16"  ? PTH_F16
                                          : dtype == "BF16" ? PTH_BF16
                                                            : PTH_OTHER;
                if (dt == PTH_OTHER || off0 < 0 || off1 < off0)
                    continue;
                if (shape.size() > PTH_MAX_DIMS)
                    bad("Tensor <%s> has rank %zu", name.c_str(), shape.size());
                struct pth_tensor t;
                memset(&t, 0, sizeof(t));
                t.ndim = (int)shape.size();
                t.dtype = dt;
                long n = 1;
                for (int d = t.ndim - 1; d >= 0; d--) {
                    t.shape[d] = shape[d];
                    t.stride[d] = n;
                    n *= shape[d];
                }
                t.data_offset = (off_t)(8 + hlen + (uint64_t)off0);
                t.storage_bytes = (size_t)(off1 - off0);
                if ((size_t)n * dtype_bytes(dt) != t.storage_bytes ||
                    (uint64_t)t.data_offset + t.storage_bytes > f.n)
                    bad("Tensor <%s> does not match its data in <%s>", name.c_str(), path);
                t.name = strdup(name.c_str());
                ts.push_back(t);
            } while (j.eat(','));
        j.expect('}');
    }
    catch (...) {
        for (auto &t : ts)
            free(t.name);
        throw;
    }
    return ts;
}

float to_float(const unsigned char *p, enum pth_dtype d)
{
    float f;
    uint32_t u;
    if (d == PTH_F32) {
        memcpy(&f, p, 4);
        return f;
    }
    const uint16_t h = (uint16_t)le(p, 2);
    if (d == PTH_BF16)
        u = (uint32_t)h << 16;
    else {
        // IEEE binary16 -> binary32, exact: rebias the exponent, widen the
        // mantissa; subnormal halves become normal floats.
        const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
        uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff;
        if (e == 31)
            u = sign | 0x7f800000u | m << 13;
        else if (e)
            u = sign | (e + 112) << 23 | m << 13;
        else if (!m)
            u = sign;
        else {
            e = 113;
            while (!(m & 0x400)) {
                m <<= 1;
                e--;
            }
            u = sign | e << 23 | (m & 0x3ff) << 13;
        }
    }
    memcpy(&f, &u, 4);
    return f;
}

bool read_exact(FILE *fp, off_t off, void *dst, size_t n)
{
    return fseeko(fp, off, SEEK_SET) == 0 && fread(dst, 1, n, fp) == n;
}

}  // namespace

extern "C" void pth_open(struct pth_file *pf, const char *path)
{
    memset(pf, 0, sizeof(*pf));
    if (pending())
        return;
    FILE *fp = fopen(path, "rb");
    if (!fp) {
        fail("Unable to open checkpoint <%s>", path);
        return;
    }
    std::vector<struct pth_tensor> ts;
    Unpickler *up = nullptr;
    try {
        const Mapped f(fp, path);
        if (f.n < 4)
            bad("<%s> is too short to be a PyTorch checkpoint", path);
        const bool zip = memcmp(f.p, "PK\003\004", 4) == 0;
        if (!zip && is_safetensors(f))
            ts = open_safetensors(f, path);
        else {
            StorageIndex ix;
            const Obj *sd = zip ? open_zip(f, path, up, ix) : open_legacy(f, path, up, ix);
            if (!sd)
                bad("No state_dict of tensors found in <%s>", path);
            ts = index_state_dict(sd, ix, path);
        }
    }
    catch (const Bad &b) {
        delete up;
        for (auto &t : ts)
            free(t.name);
        fclose(fp);
        fail("%s", b.msg.c_str());
        return;
    }
    delete up;
    pf->fp = fp;
    pf->path = strdup(path);
    pf->ntensors = (int)ts.size();
    pf->tensors = (struct pth_tensor *)malloc(ts.size() * sizeof(ts[0]) + 1);
    if (!ts.empty())
        memcpy(pf->tensors, ts.data(), ts.size() * sizeof(ts[0]));
}

extern "C" const struct pth_tensor *pth_find(const struct pth_file *pf,
                                             const char *name)
{
    for (int i = 0; i < pf->ntensors; i++)
        if (!strcmp(pf->tensors[i].name, name))
            return &pf->tensors[i];
    return NULL;
}

extern "C" int pth_strip_prefix(struct pth_file *pf, const char *prefix)
{
    const size_t n = strlen(prefix);
    int k = 0;
    for (int i = 0; i < pf->ntensors; i++) {
        char *name = pf->tensors[i].name;
        if (!strncmp(name, prefix, n)) {
            memmove(name, name + n, strlen(name + n) + 1);
            k++;
        }
    }
    return k;
}

extern "C" const struct pth_tensor *pth_require(const struct pth_file *pf,
                                                const char *name, int ndim,
                                                const long *shape)
{
    const struct pth_tensor *t = pth_find(pf, name);
    if (pending())
        return NULL;
    if (!t) {
        fail("Tensor <%s> not found in checkpoint <%s>", name, pf->path);
        return NULL;
    }
    if (t->ndim != ndim) {
        fail("Tensor <%s> has rank %d, expected %d", name, t->ndim, ndim);
        return NULL;
    }
    for (int d = 0; d < ndim; d++)
        if (shape && shape[d] >= 0 && t->shape[d] != shape[d]) {
            fail("Tensor <%s> has size %ld along axis %d, expected %ld", name,
                 t->shape[d], d, shape[d]);
            return NULL;
        }
    return t;
}

extern "C" long pth_numel(const struct pth_tensor *t)
{
    long n = 1;
    for (int d = 0; d < t->ndim; d++)
        n *= t->shape[d];
    return n;
}

// The bytes of the tensors (not of their storages, which views share).
extern "C" double pth_bytes(const struct pth_file *pf, const char *prefix)
{
    const size_t n = strlen(prefix);
    double s = 0;
    for (int i = 0; i < pf->ntensors; i++)
        if (!strncmp(pf->tensors[i].name, prefix, n))
            s += (double)pth_numel(&pf->tensors[i]) * dtype_bytes(pf->tensors[i].dtype);
    return s;
}

// A C-contiguous float32 copy: one read for a contiguous tensor, else
// the storage is read and the view gathered in C order.
extern "C" float *pth_read_f32(const struct pth_file *pf,
                               const struct pth_tensor *t)
{
    if (pending() || !t)
        return NULL;
    if (t->dtype == PTH_OTHER) {
        fail("Tensor <%s>: not a floating-point tensor", t->name);
        return NULL;
    }
    const long n = pth_numel(t);
    const size_t es = dtype_bytes(t->dtype);
    bool contiguous = true;
    long expect = 1;
    for (int d = t->ndim - 1; d >= 0; d--) {
        if (t->shape[d] != 1 && t->stride[d] != expect)
            contiguous = false;
        expect *= t->shape[d];
    }
    const size_t span = contiguous ? (size_t)n * es : t->storage_bytes;
    const off_t at = t->data_offset + (contiguous ? (off_t)t->storage_offset * (off_t)es : 0);
    if (contiguous && (size_t)(t->storage_offset + n) * es > t->storage_bytes) {
        fail("Tensor <%s>: %ld elements do not fit its %zu bytes", t->name, n,
             t->storage_bytes);
        return NULL;
    }
    float *out = (float *)malloc((size_t)(n > 0 ? n : 1) * sizeof(float));
    std::vector<unsigned char> raw(t->dtype == PTH_F32 && contiguous ? 0 : span);
    unsigned char *dst = raw.empty() ? (unsigned char *)out : raw.data();
    if (!read_exact(pf->fp, at, dst, span)) {
        free(out);
        fail("Tensor <%s>: read failed in <%s>", t->name, pf->path);
        return NULL;
    }
    if (contiguous) {
        if (!raw.empty())
            for (long i = 0; i < n; i++)
                out[i] = to_float(raw.data() + i * es, t->dtype);
        return out;
    }
    long idx[PTH_MAX_DIMS] = {0};
    for (long i = 0; i < n; i++) {
        long off = t->storage_offset;
        for (int d = 0; d < t->ndim; d++)
            off += idx[d] * t->stride[d];
        out[i] = to_float(raw.data() + off * es, t->dtype);
        for (int d = t->ndim - 1; d >= 0; d--) {
            if (++idx[d] < t->shape[d])
                break;
            idx[d] = 0;
        }
    }
    return out;
}

extern "C" void pth_close(struct pth_file *pf)
{
    if (pf->fp)
        fclose(pf->fp);
    for (int i = 0; i < pf->ntensors; i++)
        free(pf->tensors[i].name);
    free(pf->tensors);
    free(pf->path);
    memset(pf, 0, sizeof(*pf));
}
