/*
 * tos_shard.c - row sharding of the decoder across the GPUs of one node.
 *
 * The reference runs on one CPU; this is the multi-GPU plan of the B200
 * build.  Output rows of every GEMV are independent (llm.c:329-349), so each
 * rank keeps a contiguous, equal slice of rows of every projection and the
 * ranks exchange the produced slices with all-gathers:
 *
 *   q, k, v   heads [h0, h0 + H/G) and kv heads [k0, k0 + K/G); the KV cache
 *             holds only the local kv heads, so attention is local
 *   o, down   rows [r0, r0 + dim/G) of the residual stream
 *   gate, up  rows [f0, f0 + ff/G)
 *   LM head   vocabulary rows [v0, v0 + vocab/G), then a distributed argmax
 *             over (value, index) pairs with the reference's tie rule
 *             (llm.c:1129-1140: first strict maximum, NaN never wins)
 *
 * Every row is computed by exactly the kernels and inputs of the one-GPU
 * model, and the exchanges are copies, so EXACT mode stays bit-identical
 * to the reference.  NCCL is loaded at run time (dlopen), so the library
 * loads on machines without it; only sharded models need it.
 */
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include "tos_internal.h"

typedef ncclResult_t (*pf_unique_id)(ncclUniqueId *);
typedef ncclResult_t (*pf_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
typedef ncclResult_t (*pf_all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
typedef ncclResult_t (*pf_destroy)(ncclComm_t);

static struct {
    int tried, ok;
    pf_unique_id unique_id;
    pf_init_rank init_rank;
    pf_all_gather all_gather;
    pf_destroy destroy;
} nccl;

static int nccl_load(void)
{
    if (nccl.tried) return nccl.ok ? TOS_OK : TOS_ENCCL;
    nccl.tried = 1;
    /* a copy already in the process (e.g. the one a framework loaded) first */
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return TOS_ENCCL;
    nccl.unique_id = (pf_unique_id)dlsym(h, "ncclGetUniqueId");
    nccl.init_rank = (pf_init_rank)dlsym(h, "ncclCommInitRank");
    nccl.all_gather = (pf_all_gather)dlsym(h, "ncclAllGather");
    nccl.destroy = (pf_destroy)dlsym(h, "ncclCommDestroy");
    nccl.ok = nccl.unique_id && nccl.init_rank && nccl.all_gather && nccl.destroy;
    return nccl.ok ? TOS_OK : TOS_ENCCL;
}

int tos_nccl_unique_id(void *out, size_t bytes)
{
    if (!out || bytes < NCCL_UNIQUE_ID_BYTES) return tos_set_status(TOS_EINVAL);
    int rc = nccl_load();
    if (rc) return tos_set_status(rc);
    ncclUniqueId id;
    if (nccl.unique_id(&id) != ncclSuccess) return tos_set_status(TOS_ENCCL);
    memcpy(out, &id, NCCL_UNIQUE_ID_BYTES);
    return tos_set_status(TOS_OK);
}

int tos_shard_range(int total, int unit, int world, int rank, int *begin, int *count)
{
    if (!begin || !count || total <= 0 || unit <= 0 || world <= 0 || rank < 0 || rank >= world)
        return tos_set_status(TOS_EINVAL);
    if (total % unit || (total / unit) % world) return tos_set_status(TOS_ENOTSUP);
    const int per = total / world;
    *begin = rank * per;
    *count = per;
    return tos_set_status(TOS_OK);
}

int tos_shard_plan(const tos_model_desc_t *d, int world, int rank, tos_shard_plan_t *p)
{
    if (!d || !p || d->n_heads <= 0 || d->dim <= 0 || d->dim % d->n_heads) return tos_set_status(TOS_EINVAL);
    memset(p, 0, sizeof(*p));
    p->world = world;
    p->rank = rank;
    const int hd = d->dim / d->n_heads;
    int rc = 0;
    /* heads whole; row slices in multiples of 32 so every slice keeps the
     * stage / block alignment of the one-GPU layout */
    if (!rc) rc = tos_shard_range(d->n_heads, 1, world, rank, &p->head0, &p->n_heads);
    if (!rc) rc = tos_shard_range(d->n_kv_heads, 1, world, rank, &p->kv_head0, &p->n_kv_heads);
    if (!rc) rc = tos_shard_range(d->dim, 32, world, rank, &p->row0, &p->n_rows);
    if (!rc) rc = tos_shard_range(d->ff_dim, 32, world, rank, &p->ff0, &p->n_ff);
    if (!rc) rc = tos_shard_range(d->vocab_size, 32, world, rank, &p->vocab0, &p->n_vocab);
    if (rc) return tos_set_status(rc);
    p->q_row0 = p->head0 * hd;
    p->n_q_rows = p->n_heads * hd;
    p->kv_row0 = p->kv_head0 * hd;
    p->n_kv_rows = p->n_kv_heads * hd;
    return tos_set_status(TOS_OK);
}

/* ---- communicator plumbing used by tos_model.c ---- */

int tos_nccl_comm_init(void **comm, int world, int rank, const void *id)
{
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId uid;
    memcpy(&uid, id, NCCL_UNIQUE_ID_BYTES);
    ncclComm_t c = NULL;
    if (nccl.init_rank(&c, world, uid, rank) != ncclSuccess) return TOS_ENCCL;
    *comm = c;
    return TOS_OK;
}

void tos_nccl_comm_destroy(void *comm)
{
    if (comm && nccl.ok) nccl.destroy((ncclComm_t)comm);
}

/* In-place when send == (char *)recv + rank * count * esize. */
int tos_nccl_all_gather(const void *send, void *recv, size_t count, int is_int, void *comm, cudaStream_t st)
{
    if (!nccl.ok) return TOS_ENCCL;
    ncclResult_t r = nccl.all_gather(send, recv, count, is_int ? ncclInt32 : ncclFloat32, (ncclComm_t)comm, st);
    return r == ncclSuccess ? TOS_OK : TOS_ENCCL;
}
