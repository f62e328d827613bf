"""A minimal WebAssembly binary writer for tests: types, function imports,
functions, one memory, one table, globals, exports, element and data
segments.  Function bodies are written as bytes with the helpers below."""
import struct

I32, I64, F32, F64, FUNCREF = 0x7F, 0x7E, 0x7D, 0x7C, 0x70
EMPTY = 0x40


def uleb(n: int) -> bytes:
    out = bytearray()
    while True:
        b = n & 0x7F
        n >>= 7
        if n:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def sleb(n: int) -> bytes:
    out = bytearray()
    while True:
        b = n & 0x7F
        n >>= 7
        if (n == 0 and not b & 0x40) or (n == -1 and b & 0x40):
            out.append(b)
            return bytes(out)
        out.append(b | 0x80)


def vec(items) -> bytes:
    items = list(items)
    return uleb(len(items)) + b"".join(items)


def name(s: str) -> bytes:
    b = s.encode()
    return uleb(len(b)) + b


# --------------------------------------------------------------- instructions
def op(code: int, *imm: bytes) -> bytes:
    return bytes([code]) + b"".join(imm)


def i32c(v):
    return op(0x41, sleb(v))


def i64c(v):
    return op(0x42, sleb(v))


def f32c(v):
    return op(0x43, struct.pack("<f", v))


def f64c(v):
    return op(0x44, struct.pack("<d", v))


def lget(i):
    return op(0x20, uleb(i))


def lset(i):
    return op(0x21, uleb(i))


def ltee(i):
    return op(0x22, uleb(i))


def gget(i):
    return op(0x23, uleb(i))


def gset(i):
    return op(0x24, uleb(i))


def call(f):
    return op(0x10, uleb(f))


def call_indirect(t):
    return op(0x11, uleb(t), uleb(0))


def br(d):
    return op(0x0C, uleb(d))


def br_if(d):
    return op(0x0D, uleb(d))


def br_table(labels, default):
    return op(0x0E, vec(uleb(x) for x in labels), uleb(default))


def block(bt=EMPTY):
    return op(0x02, bytes([bt]))


def loop(bt=EMPTY):
    return op(0x03, bytes([bt]))


def if_(bt=EMPTY):
    return op(0x04, bytes([bt]))


def block_t(type_index):
    """block with a function type (multi-value)."""
    return op(0x02, sleb(type_index))


ELSE, END, RETURN, DROP, SELECT, UNREACHABLE, NOP = b"\x05", b"\x0b", b"\x0f", b"\x1a", b"\x1b", b"\x00", b"\x01"


def load(code, offset=0, align=0):
    return op(code, uleb(align), uleb(offset))


def store(code, offset=0, align=0):
    return op(code, uleb(align), uleb(offset))


MEMORY_SIZE, MEMORY_GROW = b"\x3f\x00", b"\x40\x00"


def fc(sub, *imm):
    return op(0xFC, uleb(sub), *imm)


# ------------------------------------------------------------------- module
class Module:
    def __init__(self):
        self.types, self.imports, self.funcs, self.exports = [], [], [], []
        self.memory = None
        self.table = None
        self.globals, self.elems, self.datas = [], [], []

    def type(self, params, results) -> int:
        t = (tuple(params), tuple(results))
        if t not in self.types:
            self.types.append(t)
        return self.types.index(t)

    def import_func(self, module, fname, params, results) -> int:
        assert not self.funcs, "imports come before functions"
        self.imports.append((module, fname, self.type(params, results)))
        return len(self.imports) - 1

    def func(self, params, results, body: bytes, locals_=(), export=None) -> int:
        idx = len(self.imports) + len(self.funcs)
        self.funcs.append((self.type(params, results), list(locals_), body))
        if export:
            self.exports.append((export, 0, idx))
        return idx

    def global_(self, vtype, mutable, init: bytes) -> int:
        self.globals.append((vtype, mutable, init))
        return len(self.globals) - 1

    def build(self) -> bytes:
        def section(i, payload):
            return bytes([i]) + uleb(len(payload)) + payload

        out = b"\x00asm\x01\x00\x00\x00"
        out += section(1, vec(b"\x60" + vec(bytes([p]) for p in ps) + vec(bytes([r]) for r in rs)
                              for ps, rs in self.types))
        if self.imports:
            out += section(2, vec(name(m) + name(n) + b"\x00" + uleb(t) for m, n, t in self.imports))
        out += section(3, vec(uleb(t) for t, _, _ in self.funcs))
        if self.table is not None:
            out += section(4, vec([bytes([FUNCREF]) + b"\x00" + uleb(self.table)]))
        if self.memory is not None:
            lo, hi = self.memory
            lim = (b"\x00" + uleb(lo)) if hi is None else (b"\x01" + uleb(lo) + uleb(hi))
            out += section(5, vec([lim]))
        if self.globals:
            out += section(6, vec(bytes([t, int(m)]) + init + END for t, m, init in self.globals))
        if self.exports:
            out += section(7, vec(name(n) + bytes([k]) + uleb(i) for n, k, i in self.exports))
        if self.elems:
            out += section(9, vec(b"\x00" + i32c(off) + END + vec(uleb(f) for f in fs) for off, fs in self.elems))
        codes = []
        for _, locs, body in self.funcs:
            lb = vec(uleb(c) + bytes([t]) for c, t in locs)
            codes.append(uleb(len(lb) + len(body) + 1) + lb + body + END)
        out += section(10, vec(codes))
        if self.datas:
            segs = []
            for off, data in self.datas:
                if off is None:
                    segs.append(b"\x01" + vec(bytes([c]) for c in data))  # passive
                else:
                    segs.append(b"\x00" + i32c(off) + END + vec(bytes([c]) for c in data))
            out += section(11, vec(segs))
        return out
