// The back-end entry: lyth_b200_select maps a lowered kernel (a descriptor of lyth-lang's KernelIr,
// crates/lyth-lang/src/ir.rs:24-56) to a kernel class of this library or refuses it with the
// reason, as lyth_ptx::emit does (crates/lyth-ptx/src/lib.rs:48-253); lyth_b200_launch launches the
// selected class from arguments in declaration order, as Function::launch_shared takes its Arg
// slots (crates/lyth-cuda/src/lib.rs:483-549).
//
// Selection is by what the kernel computes, not by its name: the body's drained registers are
// written out as expressions over declaration slots (a load of slot 2 is L2, a parameter P1, a
// load through split views L10.0w1 -- slot 10, part 0 of a split whose width is slot 1, and so
// on outward-in), and the result has to equal the expression of a class exactly, operation for
// operation, with the parameter types in the class's order. Since the fma formation of the
// lowering (ir.rs:2388-2429) is part of the expression, a body that rounds differently from a
// class's kernel is not that class: the library never runs a kernel that would not be bit-exact
// with the evaluator for the source it was given (the bf16 contraction, which the evaluator
// computes with unfused f32 arithmetic and this library on tensor cores, is the one class whose
// contract is a tolerance, 1e-2 relative).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"

namespace lyth {
namespace {

struct ClassSpec {
    int cls;
    const char *entry;
    const char *types;    // one letter per declaration slot: U u32, F f32, B f32 buffer, H bf16 buffer
    uint32_t rank, tiled, contract;
    const char *body;     // canonical drains (sorted, ';'-joined) or the reduction
};

// Canonical bodies of the kernels this library has (the examples' bodies after lowering).
const ClassSpec kClasses[] = {
    {LYTH_CLASS_SAXPY, "saxpy", "UFBB", 1, 0, 0, "D3=(fma P1 L2 L3)"},
    {LYTH_CLASS_AXPBY, "axpby", "UFFBB", 1, 0, 0, "D4=(fma P1 L3 (mul P2 L4))"},
    {LYTH_CLASS_LERP, "lerp", "UFBBB", 1, 0, 0, "D4=(fma P1 (sub L3 L2) L2)"},
    {LYTH_CLASS_HORNER, "horner", "UFFFFBB", 1, 0, 0, "D6=(fma (fma (fma P4 L5 P3) L5 P2) L5 P1)"},
    {LYTH_CLASS_COPY2D, "copy2d", "UUBB", 2, 0, 0, "D3=L2"},
    {LYTH_CLASS_TRANSPOSE, "transpose", "UUBB", 2, 0, 0, "D3t=L2"},
    {LYTH_CLASS_TRANSPOSE_TILED, "transpose_tiled", "UUBB", 2, 1, 0, "D3t=L2"},
    {LYTH_CLASS_SUM, "sum", "UBB", 1, 0, 0, "R0(L1)>2"},
    {LYTH_CLASS_DOT, "dot", "UBBB", 1, 0, 0, "R0((mul L1 L2))>3"},
    {LYTH_CLASS_MAX, "max_of", "UBB", 1, 0, 0, "R1(L1)>2"},
    {LYTH_CLASS_MIN, "min_of", "UBB", 1, 0, 0, "R2(L1)>2"},
    {LYTH_CLASS_MATMUL_F32, "matmul", "UUUBBB", 2, 1, 1, "D5=(mul L3 L4)"},
    {LYTH_CLASS_MATMUL_BF16, "matmul_bf16", "UUUHHB", 2, 1, 1, "D5=(mul L3 L4)"},
    {LYTH_CLASS_HADAMARD_Q, "hadamard_q", "UUFBBBB", 1, 0, 0,
     "D5.0w1=(mul P2 (add L3.0w1 L3.1w1));D5.1w1=(mul P2 (sub L3.0w1 L3.1w1));"
     "D6.0w1=(mul P2 (add L4.0w1 L4.1w1));D6.1w1=(mul P2 (sub L4.0w1 L4.1w1))"},
    {LYTH_CLASS_GATE_Q, "gate_q", "UUFFFFFFFFBBBB", 1, 0, 0,
     "D12.0w1=(fma P2 L10.0w1 (fma (neg P3) L11.0w1 (fma P4 L10.1w1 (mul (neg P5) L11.1w1))));"
     "D12.1w1=(fma P6 L10.0w1 (fma (neg P7) L11.0w1 (fma P8 L10.1w1 (mul (neg P9) L11.1w1))));"
     "D13.0w1=(fma P2 L11.0w1 (fma P3 L10.0w1 (fma P4 L11.1w1 (mul P5 L10.1w1))));"
     "D13.1w1=(fma P6 L11.0w1 (fma P7 L10.0w1 (fma P8 L11.1w1 (mul P9 L10.1w1))))"},
    {LYTH_CLASS_CU_Q, "cu_q", "UUUFFFFFFFFBBBB", 1, 0, 0,
     "D13.0w1.0w2=L11.0w1.0w2;D13.0w1.1w2=L11.0w1.1w2;"
     "D13.1w1.0w2=(fma P3 L11.1w1.0w2 (fma (neg P4) L12.1w1.0w2 (fma P5 L11.1w1.1w2 (mul (neg P6) L12.1w1.1w2))));"
     "D13.1w1.1w2=(fma P7 L11.1w1.0w2 (fma (neg P8) L12.1w1.0w2 (fma P9 L11.1w1.1w2 (mul (neg P10) L12.1w1.1w2))));"
     "D14.0w1.0w2=L12.0w1.0w2;D14.0w1.1w2=L12.0w1.1w2;"
     "D14.1w1.0w2=(fma P3 L12.1w1.0w2 (fma P4 L11.1w1.0w2 (fma P5 L12.1w1.1w2 (mul P6 L11.1w1.1w2))));"
     "D14.1w1.1w2=(fma P7 L12.1w1.0w2 (fma P8 L11.1w1.0w2 (fma P9 L12.1w1.1w2 (mul P10 L11.1w1.1w2))))"},
    {LYTH_CLASS_SWAP_Q, "swap_q", "UUUBBBB", 1, 0, 0,
     "D5.0w1.0w2=L3.0w1.0w2;D5.0w1.1w2=L3.1w1.0w2;D5.1w1.0w2=L3.0w1.1w2;D5.1w1.1w2=L3.1w1.1w2;"
     "D6.0w1.0w2=L4.0w1.0w2;D6.0w1.1w2=L4.1w1.0w2;D6.1w1.0w2=L4.0w1.1w2;D6.1w1.1w2=L4.1w1.1w2"},
};

// Machines this back end accepts a kernel for: its own, and what fixtures/machine/sm_100a.json
// lists under "accepts" (a kernel written for sm_120 runs here with the retarget recorded).
const char *kOwnMachines[] = {"sm_100a", "sm_100"};
const char *kAcceptedMachines[] = {"sm_120"};

void refuse(lyth_kernel *out, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(out->message, sizeof out->message, fmt, ap);
    va_end(ap);
    out->cls = 0;
}

struct Canon {
    const lyth_ir *ir;
    std::string err;

    int param(const char *name) const {
        if (!name) return -1;
        for (uint32_t i = 0; i < ir->nparams; i++)
            if (ir->params[i].name && !strcmp(ir->params[i].name, name)) return (int)i;
        return -1;
    }
    const lyth_ir_view *view(const char *name) const {
        if (!name) return nullptr;
        for (uint32_t i = 0; i < ir->nviews; i++)
            if (ir->views[i].name && !strcmp(ir->views[i].name, name)) return &ir->views[i];
        return nullptr;
    }
    // A buffer or view as slot + split path (outermost split first).
    bool buffer(const char *name, std::string &s, int depth = 0) {
        const int p = param(name);
        if (p >= 0) {
            const int ty = ir->params[p].ty;
            if (ty != LYTH_TY_BUF_F32 && ty != LYTH_TY_BUF_F16 && ty != LYTH_TY_BUF_BF16) {
                err = std::string("`") + name + "` is read as a buffer but is a scalar parameter";
                return false;
            }
            s = std::to_string(p);
            return true;
        }
        const lyth_ir_view *v = view(name);
        if (!v || depth > 8) {
            err = std::string("no buffer or view named `") + (name ? name : "(null)") + "`";
            return false;
        }
        std::string base;
        if (!buffer(v->base, base, depth + 1)) return false;
        const int w = param(v->width);
        if (w < 0 || ir->params[w].ty != LYTH_TY_U32) {
            err = std::string("split `") + v->name + "` has no u32 width parameter";
            return false;
        }
        s = base + "." + std::to_string(v->part) + "w" + std::to_string(w);
        return true;
    }
    bool expr(int32_t reg, std::string &s, int depth = 0) {
        if (reg < 0 || (uint32_t)reg >= ir->nops || depth > 64) {
            err = "a register out of range (operands must name earlier ops)";
            return false;
        }
        const lyth_ir_op &op = ir->ops[reg];
        std::string a, b, c;
        auto operand = [&](int32_t r, std::string &o) {
            if (r >= reg) {  // SSA: an operand is defined before its use
                err = "an operand is not defined before its use";
                return false;
            }
            return expr(r, o, depth + 1);
        };
        switch (op.kind) {
            case LYTH_IR_LOAD:
                if (!buffer(op.name, a)) return false;
                s = "L" + a + (op.transposed ? "t" : "");
                return true;
            case LYTH_IR_PARAM: {
                const int p = param(op.name);
                if (p < 0 || (ir->params[p].ty != LYTH_TY_U32 && ir->params[p].ty != LYTH_TY_F32)) {
                    err = std::string("`") + (op.name ? op.name : "(null)") + "` is not a scalar parameter";
                    return false;
                }
                s = "P" + std::to_string(p);
                return true;
            }
            case LYTH_IR_CONST: {
                char buf[40];
                snprintf(buf, sizeof buf, "C%.17g", op.value);
                s = buf;
                return true;
            }
            case LYTH_IR_BIN: {
                static const char *names[] = {"add", "sub", "mul", "div", "max", "min"};
                if (op.bin < 0 || op.bin > 5) {
                    err = "an unknown binary operation";
                    return false;
                }
                if (!operand(op.a, a) || !operand(op.b, b)) return false;
                s = std::string("(") + names[op.bin] + " " + a + " " + b + ")";
                return true;
            }
            case LYTH_IR_FMA:
                if (!operand(op.a, a) || !operand(op.b, b) || !operand(op.c, c)) return false;
                s = "(fma " + a + " " + b + " " + c + ")";
                return true;
            case LYTH_IR_NEG:
                if (!operand(op.a, a)) return false;
                s = "(neg " + a + ")";
                return true;
            default:
                err = "an op this back end does not know (zipper and uasm ops are not GPU kernels here)";
                return false;
        }
    }
};

char type_letter(int ty) {
    switch (ty) {
        case LYTH_TY_U32: return 'U';
        case LYTH_TY_F32: return 'F';
        case LYTH_TY_BUF_F32: return 'B';
        case LYTH_TY_BUF_BF16: return 'H';
        case LYTH_TY_BUF_F16: return 'h';
        default: return '?';
    }
}

}  // namespace
}  // namespace lyth

using namespace lyth;

extern "C" int lyth_b200_select(const lyth_ir *ir, lyth_kernel *out) {
    if (!out) return LYTH_E_INVALID;
    memset(out, 0, sizeof *out);
    if (!ir || !ir->name) {
        refuse(out, "no kernel given");
        return LYTH_E_INVALID;
    }
    if (ir->nparams > 32 || (ir->nparams && !ir->params) || (ir->nops && !ir->ops) || (ir->ndrains && !ir->drains) ||
        (ir->nviews && !ir->views)) {
        refuse(out, "kernel `%s`: a descriptor list is missing or longer than 32 parameters", ir->name);
        return LYTH_E_INVALID;
    }
    // UnknownTarget (lib.rs:31-45): the machine line must name this back end's machine or one
    // its machine file accepts; the retarget is recorded, never silent.
    const char *mach = ir->machine ? ir->machine : "";
    bool own = false, accepted = false;
    for (const char *m : kOwnMachines) own = own || !strcmp(m, mach);
    for (const char *m : kAcceptedMachines) accepted = accepted || !strcmp(m, mach);
    if (!own && !accepted) {
        refuse(out, "kernel `%s` names machine `%s`; this back end runs sm_100a (B200) and accepts sm_120 "
                    "kernels (fixtures/machine/sm_100a.json `accepts`). Name one of them.", ir->name, mach);
        return LYTH_E_UNSUPPORTED;
    }
    out->retargeted = accepted ? 1u : 0u;
    out->nparams = ir->nparams;
    for (uint32_t i = 0; i < ir->nparams; i++) out->param_ty[i] = ir->params[i].ty;
    // NoBound (lib.rs:49-52): a rank-1 kernel's index space is bounded by a u32 extent.
    if (ir->rank <= 1) {
        bool bound = false;
        for (uint32_t i = 0; i < ir->nparams; i++) bound = bound || ir->params[i].ty == LYTH_TY_U32;
        if (!bound) {
            refuse(out, "kernel `%s` has no parameter that bounds the index space; add an `n: u32` parameter", ir->name);
            return LYTH_E_UNSUPPORTED;
        }
    }
    // NoDrain (lib.rs:53-54)
    if (ir->ndrains == 0 && ir->reduce_op < 0) {
        refuse(out, "kernel `%s` drains nothing, so it computes a value and discards it", ir->name);
        return LYTH_E_UNSUPPORTED;
    }
    // A reduction's block tree is staged in shared memory (lib.rs:124-140).
    if (ir->reduce_op >= 0 && !ir->reduce_via_smem) {
        refuse(out, "kernel `%s` reduces `reg -> dram`, and this back end folds the block in shared memory. "
                    "Declare `reg -> smem -> dram` for this target.", ir->name);
        return LYTH_E_UNSUPPORTED;
    }
    // A coarsened tile that does not contract (lib.rs:171-180).
    if ((ir->coarsen[0] || ir->coarsen[1]) && !ir->contract) {
        refuse(out, "kernel `%s` coarsens a tile that does not contract. A transpose's tiled body moves one element "
                    "per thread and holds nothing across a loop, so there is nothing for a thread to own several of.",
               ir->name);
        return LYTH_E_UNSUPPORTED;
    }
    Canon cn{ir, {}};
    std::vector<std::string> parts;
    for (uint32_t d = 0; d < ir->ndrains; d++) {
        std::string tgt, e;
        if (!cn.buffer(ir->drains[d].buffer, tgt) || !cn.expr(ir->drains[d].reg, e)) {
            refuse(out, "kernel `%s`: %s", ir->name, cn.err.c_str());
            return LYTH_E_INVALID;
        }
        parts.push_back("D" + tgt + (ir->drains[d].transposed ? "t" : "") + "=" + e);
    }
    std::sort(parts.begin(), parts.end());
    std::string body;
    for (size_t i = 0; i < parts.size(); i++) body += (i ? ";" : "") + parts[i];
    if (ir->reduce_op >= 0) {
        std::string e, into;
        if (!cn.expr(ir->reduce_reg, e) || !cn.buffer(ir->reduce_into, into)) {
            refuse(out, "kernel `%s`: %s", ir->name, cn.err.c_str());
            return LYTH_E_INVALID;
        }
        body = (body.empty() ? "" : body + ";") + "R" + std::to_string(ir->reduce_op) + "(" + e + ")>" + into;
    }
    std::string types;
    for (uint32_t i = 0; i < ir->nparams; i++) types += type_letter(ir->params[i].ty);
    // Narrow storage (ADR-0024): the streams, the transposes and the reductions also run with every
    // data buffer f16, or every one bf16 (a reduction's partials stay f32), as the f32 class.
    int storage = 0;
    std::string widened = types;
    {
        const int into = ir->reduce_op >= 0 ? cn.param(ir->reduce_into) : -1;
        bool mixed = false;
        for (uint32_t i = 0; i < ir->nparams; i++) {
            const int ty = ir->params[i].ty;
            if (ty != LYTH_TY_BUF_F16 && ty != LYTH_TY_BUF_BF16) continue;
            const int st = ty == LYTH_TY_BUF_F16 ? LYTH_NARROW_F16 : LYTH_NARROW_BF16;
            if ((int)i == into || (storage && storage != st)) mixed = true;
            storage = st;
            widened[i] = 'B';
        }
        if (mixed) storage = -1;
    }
    const uint32_t rank = ir->rank ? ir->rank : 1;
    const uint32_t tiled = (ir->tile[0] || ir->tile[1]) ? 1u : 0u;
    for (const ClassSpec &c : kClasses) {
        if (rank != c.rank || ir->contract != c.contract || body != c.body) continue;
        const bool narrow_ok = c.cls != LYTH_CLASS_MATMUL_F32 && c.cls != LYTH_CLASS_MATMUL_BF16 &&
                               c.cls != LYTH_CLASS_HADAMARD_Q && c.cls != LYTH_CLASS_GATE_Q && c.cls != LYTH_CLASS_CU_Q &&
                               c.cls != LYTH_CLASS_SWAP_Q && c.cls != LYTH_CLASS_TRANSPOSE;
        int st = 0;
        if (types == c.types) st = 0;
        else if (storage > 0 && narrow_ok && widened == c.types) st = storage;
        else continue;
        if (c.cls == LYTH_CLASS_TRANSPOSE || c.cls == LYTH_CLASS_TRANSPOSE_TILED) {
            if (tiled != c.tiled) continue;
        }
        out->cls = c.cls;
        out->storage = st;
        snprintf(out->entry, sizeof out->entry, "%s%s", c.entry, st == LYTH_NARROW_F16 ? "_f16" : (st == LYTH_NARROW_BF16 ? "_bf16" : ""));
        for (uint32_t i = 0; i < ir->nparams && i < 16; i++) out->slot[i] = (int32_t)i;
        if (out->retargeted)
            snprintf(out->message, sizeof out->message, "kernel `%s` written for `%s`, run as %s on sm_100a (retarget "
                                                        "accepted by fixtures/machine/sm_100a.json)", ir->name, mach, c.entry);
        return LYTH_OK;
    }
    refuse(out, "kernel `%s` computes a body this back end has no kernel for (%s over %s): the B200 back end "
                "covers the streamed elementwise, transpose, reduction, contraction and state-vector gate classes "
                "bit for bit; it does not emit a generic kernel",
           ir->name, body.size() > 160 ? (body.substr(0, 157) + "...").c_str() : body.c_str(), types.c_str());
    return LYTH_E_UNSUPPORTED;
}

extern "C" size_t lyth_b200_workspace_bytes(const lyth_kernel *k, void *const *args) {
    (void)args;
    if (!k || !k->cls) return 0;
    return 0;  // every class writes only the caller's buffers (reductions: the `into` partials)
}

extern "C" int lyth_b200_launch(const lyth_kernel *k, void *const *args, const lyth_launch *launch, cudaStream_t s) {
    if (!k || !k->cls || !args) return LYTH_E_INVALID;
    for (uint32_t i = 0; i < k->nparams; i++)
        if (!args[i]) return LYTH_E_INVALID;
    auto u = [&](int i) { return *static_cast<const uint32_t *>(args[i]); };
    auto f = [&](int i) { return *static_cast<const float *>(args[i]); };
    auto bf = [&](int i) { return reinterpret_cast<float *>(*static_cast<const uint64_t *>(args[i])); };
    auto bh = [&](int i) { return reinterpret_cast<uint16_t *>(*static_cast<const uint64_t *>(args[i])); };
    auto m8 = [&](int i0, float *m) {
        for (int j = 0; j < 8; j++) m[j] = f(i0 + j);
    };
    float m[8];
    if (k->storage > 0) {
        auto bn = [&](int i) { return reinterpret_cast<uint16_t *>(*static_cast<const uint64_t *>(args[i])); };
        const int ty = k->storage;
        float c[4];
        switch (k->cls) {
            case LYTH_CLASS_SAXPY: c[0] = f(1); return lyth_b200_stream_narrow(LYTH_STREAM_SAXPY, ty, u(0), c, bn(2), bn(3), bn(3), s);
            case LYTH_CLASS_AXPBY:
                c[0] = f(1); c[1] = f(2);
                return lyth_b200_stream_narrow(LYTH_STREAM_AXPBY, ty, u(0), c, bn(3), bn(4), bn(4), s);
            case LYTH_CLASS_LERP: c[0] = f(1); return lyth_b200_stream_narrow(LYTH_STREAM_LERP, ty, u(0), c, bn(2), bn(3), bn(4), s);
            case LYTH_CLASS_HORNER:
                for (int i = 0; i < 4; i++) c[i] = f(1 + i);
                return lyth_b200_stream_narrow(LYTH_STREAM_HORNER, ty, u(0), c, bn(5), nullptr, bn(6), s);
            case LYTH_CLASS_COPY2D:
                return lyth_b200_stream_narrow(LYTH_STREAM_COPY, ty, (uint64_t)u(0) * u(1), nullptr, bn(2), nullptr, bn(3), s);
            case LYTH_CLASS_TRANSPOSE_TILED: return lyth_b200_transpose_narrow(ty, u(0), u(1), bn(2), bn(3), s);
            case LYTH_CLASS_SUM:
            case LYTH_CLASS_MAX:
            case LYTH_CLASS_MIN: {
                const int op = k->cls == LYTH_CLASS_SUM ? 0 : (k->cls == LYTH_CLASS_MAX ? 1 : 2);
                const uint32_t grid = launch && launch->grid ? launch->grid : lyth_b200_reduce_grid(u(0));
                return lyth_b200_reduce_partials_narrow(op, ty, u(0), bn(1), nullptr, grid, bf(2), s);
            }
            case LYTH_CLASS_DOT: {
                const uint32_t grid = launch && launch->grid ? launch->grid : lyth_b200_reduce_grid(u(0));
                return lyth_b200_reduce_partials_narrow(0, ty, u(0), bn(1), bn(2), grid, bf(3), s);
            }
            default: return LYTH_E_UNSUPPORTED;
        }
    }
    switch (k->cls) {
        case LYTH_CLASS_SAXPY: return lyth_b200_saxpy(u(0), f(1), bf(2), bf(3), s);
        case LYTH_CLASS_AXPBY: return lyth_b200_axpby(u(0), f(1), f(2), bf(3), bf(4), s);
        case LYTH_CLASS_LERP: return lyth_b200_lerp(u(0), f(1), bf(2), bf(3), bf(4), s);
        case LYTH_CLASS_HORNER: return lyth_b200_horner(u(0), f(1), f(2), f(3), f(4), bf(5), bf(6), s);
        case LYTH_CLASS_COPY2D: return lyth_b200_copy2d(u(0), u(1), bf(2), bf(3), s);
        case LYTH_CLASS_TRANSPOSE: return lyth_b200_transpose_naive(u(0), u(1), bf(2), bf(3), s);
        case LYTH_CLASS_TRANSPOSE_TILED: return lyth_b200_transpose_tiled(u(0), u(1), bf(2), bf(3), s);
        case LYTH_CLASS_SUM:
        case LYTH_CLASS_MAX:
        case LYTH_CLASS_MIN: {
            const int op = k->cls == LYTH_CLASS_SUM ? 0 : (k->cls == LYTH_CLASS_MAX ? 1 : 2);
            const uint32_t grid = launch && launch->grid ? launch->grid : lyth_b200_reduce_grid(u(0));
            return lyth_b200_reduce_partials(op, u(0), bf(1), nullptr, grid, bf(2), s);
        }
        case LYTH_CLASS_DOT: {
            const uint32_t grid = launch && launch->grid ? launch->grid : lyth_b200_reduce_grid(u(0));
            return lyth_b200_reduce_partials(0, u(0), bf(1), bf(2), grid, bf(3), s);
        }
        case LYTH_CLASS_MATMUL_F32: return lyth_b200_matmul_f32(u(0), u(1), u(2), bf(3), bf(4), bf(5), 1, s);
        case LYTH_CLASS_MATMUL_BF16: return lyth_b200_matmul_bf16(u(0), u(1), u(2), bh(3), bh(4), bf(5), s);
        case LYTH_CLASS_HADAMARD_Q: return lyth_b200_hadamard(u(0), u(1), f(2), bf(3), bf(4), bf(5), bf(6), s);
        case LYTH_CLASS_GATE_Q: m8(2, m); return lyth_b200_gate(u(0), u(1), m, bf(10), bf(11), bf(12), bf(13), s);
        case LYTH_CLASS_CU_Q: m8(3, m); return lyth_b200_cu(u(0), u(1), u(2), m, bf(11), bf(12), bf(13), bf(14), s);
        case LYTH_CLASS_SWAP_Q: return lyth_b200_swap(u(0), u(1), u(2), bf(3), bf(4), bf(5), bf(6), s);
        default: return LYTH_E_UNSUPPORTED;
    }
}
