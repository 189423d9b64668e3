/*
 * atlas_data.h -- C ABI of the BOS-aligned best-fit row packer (host code).
 *
 * Replaces the packing loop of data_loader (rkstgr/atlas-jax,
 * atlas_jax/data.py:54-121).  Each row of capacity seq_len + 1 is filled by
 * repeatedly taking, from a buffer of tokenised documents, the LARGEST document
 * that fits entirely (the earliest-buffered one among equal lengths); when none
 * fits, the SHORTEST document (earliest among equals) is cropped to the remaining
 * space and its tail discarded.  Rows are therefore 100% utilised and start with a
 * document's first token (BOS, when the caller prepends it as the reference's
 * tokenizer.encode(prepend=bos) does).  A batch is (batch_size, seq_len) inputs =
 * row[:-1] and targets = row[1:], int32, row-major.
 *
 * Feeding: the reference refills its buffer to buffer_size documents before every
 * placement (data.py:94-95).  Here the caller pushes documents; when a placement
 * would need a buffer of buffer_size documents and fewer are held,
 * atlas_packer_next_batch returns ATLAS_PACK_NEED_DOCS with its progress kept, and
 * the caller pushes more and calls again.  Results are identical to the
 * reference's for the same document stream.
 *
 * A packer is not thread-safe; use one per thread (one per data-parallel rank, as
 * the reference's rank/world_size sharding does).
 */
#ifndef ATLAS_DATA_H_
#define ATLAS_DATA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* returned by atlas_packer_next_batch when more documents are needed */
#define ATLAS_PACK_NEED_DOCS 6

typedef struct AtlasPacker AtlasPacker;

/* NULL on invalid sizes (batch_size, seq_len, buffer_size must be positive). */
AtlasPacker* atlas_packer_create(int32_t batch_size, int32_t seq_len, int32_t buffer_size);
void atlas_packer_destroy(AtlasPacker* p);

/* Appends ndocs documents, document i = tokens[offsets[i] .. offsets[i+1]) (offsets
 * has ndocs + 1 entries, increasing).  Documents must be non-empty (the reference's
 * always start with BOS; an empty one would make its crop step fail).  Returns
 * ATLAS_OK or ATLAS_ERR_INVALID_ARGUMENT (nothing appended). */
int atlas_packer_push(AtlasPacker* p, const int32_t* tokens, const int64_t* offsets, int64_t ndocs);

/* Documents currently buffered. */
int64_t atlas_packer_buffered(const AtlasPacker* p);

/* Fills inputs and targets (batch_size x seq_len int32 each) with the next batch.
 * Returns ATLAS_OK, or ATLAS_PACK_NEED_DOCS (nothing written; push and retry). */
int atlas_packer_next_batch(AtlasPacker* p, int32_t* inputs, int32_t* targets);

#ifdef __cplusplus
}
#endif

#endif /* ATLAS_DATA_H_ */
