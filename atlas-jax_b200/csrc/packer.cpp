// BOS-aligned best-fit row packer (include/atlas_data.h), host code.
// Restates the packing loop of atlas_jax/data.py:54-121 with an ordered index
// instead of the reference's linear scans: documents are keyed by (length,
// arrival sequence), so "largest that fits, earliest among equals" and "shortest,
// earliest among equals" are O(log n) lookups and buffer order never has to be
// maintained explicitly (the reference's list.pop keeps arrival order).
#include <cstring>
#include <iterator>
#include <map>
#include <set>
#include <utility>
#include <vector>

#include "atlas_data.h"
#include "atlas_scan.h"

struct AtlasPacker {
  int32_t B, T, buffer_size;
  int64_t seq = 0;
  std::map<int64_t, std::vector<int32_t>> docs;  // arrival sequence -> tokens
  std::set<std::pair<int64_t, int64_t>> index;    // (length, arrival sequence)
  std::vector<int32_t> rows;                      // B x (T + 1), the batch in progress
  int32_t row = 0, pos = 0;                       // progress inside it
};

extern "C" {

AtlasPacker* atlas_packer_create(int32_t batch_size, int32_t seq_len, int32_t buffer_size) {
  if (batch_size <= 0 || seq_len <= 0 || buffer_size <= 0) return nullptr;
  AtlasPacker* p = new AtlasPacker;
  p->B = batch_size;
  p->T = seq_len;
  p->buffer_size = buffer_size;
  p->rows.assign((size_t)batch_size * (seq_len + 1), 0);
  return p;
}

void atlas_packer_destroy(AtlasPacker* p) { delete p; }

int atlas_packer_push(AtlasPacker* p, const int32_t* tokens, const int64_t* offsets, int64_t ndocs) {
  if (!p || ndocs < 0 || (ndocs > 0 && (!tokens || !offsets))) return ATLAS_ERR_INVALID_ARGUMENT;
  for (int64_t i = 0; i < ndocs; ++i)
    if (offsets[i + 1] <= offsets[i] || offsets[i] < 0) return ATLAS_ERR_INVALID_ARGUMENT;
  for (int64_t i = 0; i < ndocs; ++i) {
    const int64_t n = offsets[i + 1] - offsets[i];
    p->docs.emplace(p->seq, std::vector<int32_t>(tokens + offsets[i], tokens + offsets[i + 1]));
    p->index.emplace(n, p->seq);
    ++p->seq;
  }
  return ATLAS_OK;
}

int64_t atlas_packer_buffered(const AtlasPacker* p) { return p ? (int64_t)p->docs.size() : 0; }

int atlas_packer_next_batch(AtlasPacker* p, int32_t* inputs, int32_t* targets) {
  if (!p || !inputs || !targets) return ATLAS_ERR_INVALID_ARGUMENT;
  const int32_t cap = p->T + 1;  // data.py:82 row_capacity
  while (p->row < p->B) {
    int32_t* r = p->rows.data() + (size_t)p->row * cap;
    while (p->pos < cap) {
      if ((int64_t)p->docs.size() < p->buffer_size) return ATLAS_PACK_NEED_DOCS;  // data.py:94-95
      const int64_t remaining = cap - p->pos;
      // largest length <= remaining, earliest arrival among equals (data.py:100-106)
      auto it = p->index.upper_bound({remaining, INT64_MAX});
      if (it != p->index.begin()) {
        const int64_t len = std::prev(it)->first;
        it = p->index.lower_bound({len, INT64_MIN});
        auto d = p->docs.find(it->second);
        std::memcpy(r + p->pos, d->second.data(), (size_t)len * sizeof(int32_t));
        p->pos += (int32_t)len;
        p->docs.erase(d);
        p->index.erase(it);
      } else {  // nothing fits: crop the shortest, earliest among equals (data.py:113-117)
        it = p->index.begin();
        auto d = p->docs.find(it->second);
        std::memcpy(r + p->pos, d->second.data(), (size_t)remaining * sizeof(int32_t));
        p->pos += (int32_t)remaining;
        p->docs.erase(d);
        p->index.erase(it);
      }
    }
    ++p->row;
    p->pos = 0;
  }
  for (int32_t b = 0; b < p->B; ++b) {  // data.py:119-120: inputs row[:-1], targets row[1:]
    const int32_t* r = p->rows.data() + (size_t)b * cap;
    std::memcpy(inputs + (size_t)b * p->T, r, (size_t)p->T * sizeof(int32_t));
    std::memcpy(targets + (size_t)b * p->T, r + 1, (size_t)p->T * sizeof(int32_t));
  }
  p->row = 0;
  return ATLAS_OK;
}

}  // extern "C"
