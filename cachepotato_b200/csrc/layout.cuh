// layout.cuh — the K-permutation shared by the expert kernels and their activation writers.
//
// The expert kernels feed m16n8k16 tensor-core MMAs straight from Q4_0 / Q8_0 groups as they
// sit in a CPW1 v4 file (18- / 34-byte groups, so no 16-byte structure lines up with a group).
// Within each 64-value group pair the four threads of an MMA quad read 32-bit words that are
// aligned and bank-conflict free; which values a word holds fixes which K slot of the MMA each
// value must occupy. The reduction order of a dot product does not matter to the result's
// meaning, so the activation operand is stored PERMUTED the same way: position
//     pos = 16*t + 4*s + i      (t = thread in quad, s = k16 step, i = slot in [2t,2t+1,2t+8,2t+9])
// of each 64-block holds element pos_to_elem[pos] of that block. One thread's B fragments for
// a whole group pair are then 32 contiguous bytes (two 16-byte loads).
#pragma once
#include <stdint.h>

#include "cpg.h"

namespace cpg {

struct Perm64 {
    uint8_t pos_to_elem[64];
    uint8_t elem_to_pos[64];
};

// quant-byte indices (within a group's 16 / 32 payload bytes) held by word `w` of thread t
// w = 0,1 for group j (first of the pair), 2,3 for group j+1
constexpr int q4_byte(int t, int w, int b) {
    // Q4 group pair = 9 words: w0 = [s_j, q_j0, q_j1], w1..w3 = q_j[2..13], w4 = [q_j14, q_j15, s_j+1],
    // w5..w8 = q_j+1[0..15]. Thread t reads w(1+t) and w(5+t); thread 3 rebuilds [q0,q1,q14,q15].
    return w == 0 ? (t < 3 ? 4 * t + 2 + b : (b < 2 ? b : 12 + b)) : 4 * t + b;
}
constexpr int q8_byte(int t, int w, int b) {
    // Q8 group pair = 17 words: w0 = [s_j, q_j0, q_j1], w1..w7 = q_j[2..29], w8 = [q_j30, q_j31,
    // s_j+1], w9..w16 = q_j+1[0..31]. Thread t reads w(1+t), w(5+t) (thread 3 rebuilds
    // [q0,q1,q30,q31] from w0,w8), w(9+t), w(13+t).
    return w == 0 ? 4 * t + 2 + b
         : w == 1 ? (t < 3 ? 4 * t + 18 + b : (b < 2 ? b : 28 + b))
         : w == 2 ? 4 * t + b
                  : 4 * t + 16 + b;
}

constexpr Perm64 make_perm(int enc) {
    Perm64 p{};
    for (int t = 0; t < 4; ++t)
        for (int s = 0; s < 4; ++s)
            for (int i = 0; i < 4; ++i) {
                int e = 0;
                if (enc == CPG_ENC_Q4) {
                    // step s uses word s/2 of its group: sub-step 0 takes bytes (b0,b2), 1 takes (b1,b3);
                    // slots i = 0,1 are low nibbles (elements c), i = 2,3 high nibbles (c + 16)
                    const int w = s / 2, sub = s % 2;
                    const int b = (i % 2 == 0 ? 0 : 2) + sub;
                    e = q4_byte(t, w, b) + (i >= 2 ? 16 : 0) + (w ? 32 : 0);
                } else {
                    // step s is word s of the pair; slots i = bytes b0..b3 of that word
                    e = q8_byte(t, s, i) + (s >= 2 ? 32 : 0);
                }
                p.pos_to_elem[16 * t + 4 * s + i] = (uint8_t)e;
            }
    for (int i = 0; i < 64; ++i) p.elem_to_pos[p.pos_to_elem[i]] = (uint8_t)i;
    return p;
}

constexpr Perm64 kPermQ4 = make_perm(CPG_ENC_Q4);
constexpr Perm64 kPermQ8 = make_perm(CPG_ENC_Q8);

}  // namespace cpg
