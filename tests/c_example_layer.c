/* One rank of an SP group of S on device `dev`; peer buffers were exchanged with
 * fu_buffer_export / fu_buffer_import (their pointers as mapped in this process).
 * For brevity the contexts live for one layer call here; in practice create them
 * once per rank and reuse them for every call. */
#include "flash_ulysses_b200.h"

int layer(int dev, int S, int me, void* const* q_recv, void* const* k_recv,
          void* const* v_recv, uint32_t* const* sync, void* const* gather,
          uint32_t* const* o_sync, const void* x, const void* w_qkv, const int64_t* pos,
          const float* q_gamma, const float* k_gamma, const float* rope, int64_t rope_rows,
          const void* attn, const void* w_o, void* out, int64_t L, void* stream) {
    fu_qkv_topology t = {0};
    t.device = dev; t.sp_size = S; t.sp_rank = me;
    t.q_heads = 32; t.kv_heads = 8; t.hidden_size = 4096; t.capacity_rows = S * 4096;
    for (int d = 0; d < S; ++d) {
        t.q_recv[d] = q_recv[d]; t.k_recv[d] = k_recv[d]; t.v_recv[d] = v_recv[d];
        t.sync[d] = sync[d];
    }
    fu_qkv_ctx* qkv = NULL;
    if (fu_qkv_create(&t, &qkv) != FU_OK) return -1;          /* fu_last_error() says why */
    int rc = fu_qkv_forward(qkv, x, w_qkv, pos, q_gamma, k_gamma, rope, L, rope_rows,
                            1e-6, 1e-6, 0, stream, NULL);
    /* ... attention over q_recv/k_recv/v_recv[me] writes attn [S*L, 32/S*128] ... */
    fu_oproj_topology o = {0};
    o.device = dev; o.sp_size = S; o.sp_rank = me;
    o.q_heads = 32; o.hidden_size = 4096; o.max_local_tokens = 4096;
    for (int d = 0; d < S; ++d) { o.gather[d] = gather[d]; o.sync[d] = o_sync[d]; }
    fu_oproj_ctx* op = NULL;
    if (rc == FU_OK && fu_oproj_create(&o, &op) == FU_OK)
        rc = fu_oproj_forward(op, attn, w_o, L, out, 0, stream);   /* out [L, 4096] */
    fu_oproj_destroy(op);
    fu_qkv_destroy(qkv);
    return rc;
}
