// Paged KV-cache bookkeeping in C++: page pool with reference counts,
// per-sequence page lists, zero-copy prefix sharing and copy-on-write forks.
//
// Replaces the reference's KV handling by tensor copies -- HF DynamicCache
// `repeat_interleave` for prefix de-duplication and `crop` for truncation
// (src/inference_scaling/arllm/backends/transformers_backend.py:368-416) and the
// block-grown cache (growing_cache.py:12-82) -- with page tables: sequences
// that share a prefix share its pages, a suffix-MH proposal forks a chain at
// its cut (only a partially filled last page is copied), and rejected or
// finished sequences return their pages.  The device kernels read the page
// tables this class produces.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace osb {

class KVManager {
 public:
  KVManager(int num_pages, int page_size);

  int page_size() const { return page_size_; }
  int num_pages() const { return static_cast<int>(ref_.size()); }
  int free_pages() const { return static_cast<int>(free_.size()); }

  // Create an empty sequence and return its id.
  int64_t create();
  // Drop a sequence and release its pages.
  void release(int64_t seq);
  // Number of tokens whose KV slots the sequence holds.
  int length(int64_t seq) const;
  // Reserve slots for `n` more tokens; returns their physical slot ids
  // (page * page_size + offset).  Throws std::runtime_error when out of pages.
  std::vector<int32_t> append(int64_t seq, int n);
  // Shrink to `n` tokens (releasing pages no longer used).
  void truncate(int64_t seq, int n);
  // New sequence sharing the first `n` tokens of `seq`.  Full pages are shared
  // by reference; a partially filled boundary page is duplicated.  The copy
  // (src page, dst page, token count) is appended to `copies` for the device.
  int64_t fork(int64_t seq, int n, std::vector<int32_t>& copies);
  // Page list of a sequence.
  const std::vector<int32_t>& pages(int64_t seq) const;
  // Write the page table rows of `seqs` into `out` (row stride `stride`,
  // unused entries set to 0).
  void fill_table(const std::vector<int64_t>& seqs, int32_t* out, int stride) const;
  int refcount(int page) const { return ref_.at(page); }
  // New sequence made of existing pages (each gains a reference), `length` tokens.
  int64_t adopt(const std::vector<int32_t>& pages, int length);
  // Extra references held by an external owner (e.g. a prefix cache).
  void retain(int32_t page);
  void drop(int32_t page) { drop_page(page); }

 private:
  struct Seq {
    std::vector<int32_t> pages;
    int length = 0;
  };
  int32_t take_page();
  void drop_page(int32_t p);
  Seq& get(int64_t seq);
  const Seq& get(int64_t seq) const;

  int page_size_;
  std::vector<int32_t> ref_;
  std::vector<int32_t> free_;
  std::unordered_map<int64_t, Seq> seqs_;
  int64_t next_id_ = 0;
};

}  // namespace osb
