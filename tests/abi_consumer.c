/* A plain C consumer of include/sam3_b200.h, built by tests/test_abi_consumer.py both as C99 and as
 * C++14 (the language of sam3.cpp) and linked against libsam3_b200.so: the header is usable from
 * either language, the node record has one layout in both, and the host-only entries behave the
 * same as through the Python bindings.  Needs no GPU; with one present it only opens and closes a
 * backend. */
#include "sam3_b200.h"

#include <stddef.h>
#include <stdio.h>
#include <string.h>

static int failures = 0;

static void expect(int cond, const char *what) {
    if (!cond) {
        fprintf(stderr, "FAILED: %s (last error: %s)\n", what, sam3b200_last_error());
        ++failures;
    }
}

static void packed(sam3b200_tensor *t, int type, int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3,
                   size_t elt, void *data) {
    memset(t, 0, sizeof *t);
    t->type = type;
    t->ne[0] = ne0;
    t->ne[1] = ne1;
    t->ne[2] = ne2;
    t->ne[3] = ne3;
    t->nb[0] = elt;
    t->nb[1] = elt * (size_t)ne0;
    t->nb[2] = t->nb[1] * (size_t)ne1;
    t->nb[3] = t->nb[2] * (size_t)ne2;
    t->data = data;
}

int main(void) {
    void *const dev = (void *)(uintptr_t)(1u << 20); /* never dereferenced: host-only checks */
    sam3b200_tensor w, x, y, k, img, conv, odd;
    sam3b200_tensor *nodes[1];
    sam3b200_backend *be;

    expect(sizeof(sam3b200_tensor) == 192 && offsetof(sam3b200_tensor, src) == 144, "node layout");

    /* MUL_MAT over a Q8_0 [256, 96] weight: 34-byte blocks of 32 */
    packed(&w, SAM3B200_TYPE_Q8_0, 256, 96, 1, 1, 34, NULL);
    w.nb[1] = 34 * 8;
    w.nb[2] = w.nb[1] * 96;
    w.nb[3] = w.nb[2];
    packed(&x, SAM3B200_TYPE_F32, 256, 40, 1, 1, 4, dev);
    packed(&y, SAM3B200_TYPE_F32, 96, 40, 1, 1, 4, dev);
    y.op = SAM3B200_OP_MUL_MAT;
    y.src[0] = &w;
    y.src[1] = &x;
    expect(sam3b200_supports_op(&y) == 1, "MUL_MAT Q8_0 supported");
    nodes[0] = &y;
    expect(sam3b200_graph_compute(NULL, nodes, 1) == SAM3B200_STATUS_FAILED, "MUL_MAT without a weight handle");
    expect(strstr(sam3b200_last_error(), "no handle") != NULL, "names the missing weight handle");

    /* CONV_2D 3x3, pad 1: passes every check, then meets the missing backend */
    packed(&k, SAM3B200_TYPE_F16, 3, 3, 8, 16, 2, dev);
    packed(&img, SAM3B200_TYPE_F32, 20, 18, 8, 1, 4, dev);
    packed(&conv, SAM3B200_TYPE_F32, 20, 18, 16, 1, 4, dev);
    conv.op = SAM3B200_OP_CONV_2D;
    conv.src[0] = &k;
    conv.src[1] = &img;
    conv.op_params[0] = conv.op_params[1] = conv.op_params[2] = conv.op_params[3] = 1;
    conv.op_params[4] = conv.op_params[5] = 1;
    expect(sam3b200_supports_op(&conv) == 1, "CONV_2D supported");
    nodes[0] = &conv;
    expect(sam3b200_graph_compute(NULL, nodes, 1) == SAM3B200_STATUS_FAILED, "null backend refused");
    expect(strstr(sam3b200_last_error(), "null backend") != NULL, "a valid graph reaches the backend check");

    /* an op this backend does not execute */
    packed(&odd, SAM3B200_TYPE_F32, 4, 1, 1, 1, 4, dev);
    odd.op = 99;
    expect(sam3b200_supports_op(&odd) == 0, "unknown op refused");
    nodes[0] = &odd;
    expect(sam3b200_graph_compute(NULL, nodes, 1) == SAM3B200_STATUS_FAILED, "unknown op graph refused");
    expect(strstr(sam3b200_last_error(), "node 0 rejected") != NULL, "names the node");

    /* the tracker's host-side memory of one object: 9 frames (frame 0 prompted), 7 slots kept */
    {
        enum { H = 4, MD = 64, D = 256 };
        static float feats[H * H * MD], ptr[D], prompt[(7 * H * H + 16 * 4) * MD], pos[(7 * H * H + 16 * 4) * MD];
        sam3b200_mem_prompt_hparams hp = {D, MD, 7, 16};
        sam3b200_mem_bank *bank = sam3b200_mem_bank_create(&hp, H);
        int32_t frames[16], cond[16], pframes[16], n_ptrs = 0, n_ptr_tokens = 0;
        int f, ns;
        int64_t m;
        expect(bank != NULL, "mem_bank_create");
        for (f = 0; bank && f < 9; ++f) {
            feats[0] = (float)f;
            ptr[0] = (float)f;
            expect(sam3b200_mem_bank_add_slot(bank, feats, f, f == 0) == SAM3B200_STATUS_SUCCESS, "add_slot");
            expect(sam3b200_mem_bank_add_ptr(bank, ptr, f) == SAM3B200_STATUS_SUCCESS, "add_ptr");
        }
        ns = bank ? sam3b200_mem_bank_state(bank, frames, cond, 16, pframes, 16, &n_ptrs) : -1;
        expect(ns == 7 && frames[0] == 0 && cond[0] == 1 && frames[1] == 3 && frames[6] == 8 && n_ptrs == 9,
               "bank keeps the prompted frame and the newest six");
        m = bank ? sam3b200_mem_bank_prompt(bank, 9, NULL, NULL, NULL, prompt, pos, 7 * H * H + 16 * 4,
                                            &n_ptr_tokens)
                 : -1;
        expect(m == 7 * H * H + 9 * 4 && n_ptr_tokens == 9 * 4, "prompt of 7 slots and 9 pointers");
        expect(prompt[0] == 0.0f && prompt[H * H * MD] == 3.0f, "slot features in bank order");
        sam3b200_mem_bank_free(bank);
    }

    /* backend lifetime: NULL and a message without a GPU; open/close with one */
    be = sam3b200_backend_init(0);
    if (be) {
        expect(sam3b200_backend_synchronize(be) == SAM3B200_STATUS_SUCCESS, "synchronize");
        sam3b200_backend_free(be);
    } else {
        expect(sam3b200_last_error()[0] != '\0', "backend_init failure message");
    }
    expect(sam3b200_backend_synchronize(NULL) == SAM3B200_STATUS_FAILED, "null backend synchronize");

    if (failures) return 1;
    printf("ok\n");
    return 0;
}
