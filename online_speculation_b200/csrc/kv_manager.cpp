// Paged KV-cache bookkeeping (see kv_manager.h).
#include "kv_manager.h"

#include <algorithm>
#include <string>

namespace osb {

KVManager::KVManager(int num_pages, int page_size) : page_size_(page_size) {
  if (num_pages <= 0 || page_size <= 0) throw std::invalid_argument("positive page count and size required");
  ref_.assign(num_pages, 0);
  free_.reserve(num_pages);
  // hand out low page ids first
  for (int p = num_pages - 1; p >= 0; --p) free_.push_back(p);
}

int32_t KVManager::take_page() {
  if (free_.empty()) throw std::runtime_error("KV cache out of pages");
  const int32_t p = free_.back();
  free_.pop_back();
  ref_[p] = 1;
  return p;
}

void KVManager::drop_page(int32_t p) {
  if (p < 0 || p >= static_cast<int32_t>(ref_.size()) || ref_[p] <= 0)
    throw std::logic_error("page reference count underflow");
  if (--ref_[p] == 0) free_.push_back(p);
}

KVManager::Seq& KVManager::get(int64_t seq) {
  auto it = seqs_.find(seq);
  if (it == seqs_.end()) throw std::out_of_range("unknown sequence " + std::to_string(seq));
  return it->second;
}

const KVManager::Seq& KVManager::get(int64_t seq) const {
  auto it = seqs_.find(seq);
  if (it == seqs_.end()) throw std::out_of_range("unknown sequence " + std::to_string(seq));
  return it->second;
}

int64_t KVManager::create() {
  const int64_t id = next_id_++;
  seqs_.emplace(id, Seq{});
  return id;
}

void KVManager::release(int64_t seq) {
  Seq& s = get(seq);
  for (int32_t p : s.pages) drop_page(p);
  seqs_.erase(seq);
}

int KVManager::length(int64_t seq) const { return get(seq).length; }

std::vector<int32_t> KVManager::append(int64_t seq, int n) {
  if (n < 0) throw std::invalid_argument("negative append");
  Seq& s = get(seq);
  const int need_pages = (s.length + n + page_size_ - 1) / page_size_;
  const int extra = need_pages - static_cast<int>(s.pages.size());
  if (extra > static_cast<int>(free_.size())) throw std::runtime_error("KV cache out of pages");
  // A shared, partially filled last page must become private before a write.
  if (s.length % page_size_ != 0 && !s.pages.empty() && ref_[s.pages.back()] > 1)
    throw std::logic_error("append into a shared page; fork() must copy the boundary page");
  for (int i = 0; i < extra; ++i) s.pages.push_back(take_page());
  std::vector<int32_t> slots(n);
  for (int i = 0; i < n; ++i) {
    const int pos = s.length + i;
    slots[i] = s.pages[pos / page_size_] * page_size_ + pos % page_size_;
  }
  s.length += n;
  return slots;
}

void KVManager::truncate(int64_t seq, int n) {
  Seq& s = get(seq);
  if (n < 0 || n > s.length) throw std::invalid_argument("truncate beyond sequence length");
  const int keep = (n + page_size_ - 1) / page_size_;
  while (static_cast<int>(s.pages.size()) > keep) {
    drop_page(s.pages.back());
    s.pages.pop_back();
  }
  s.length = n;
}

int64_t KVManager::fork(int64_t seq, int n, std::vector<int32_t>& copies) {
  const Seq& src = get(seq);
  if (n < 0 || n > src.length) throw std::invalid_argument("fork beyond sequence length");
  const int full = n / page_size_;
  const int rem = n % page_size_;
  if (rem && free_.empty()) throw std::runtime_error("KV cache out of pages");
  Seq dst;
  dst.pages.reserve(full + 1);
  for (int i = 0; i < full; ++i) {
    const int32_t p = src.pages[i];
    ++ref_[p];
    dst.pages.push_back(p);
  }
  if (rem) {
    const int32_t from = src.pages[full];
    const int32_t to = take_page();
    dst.pages.push_back(to);
    copies.push_back(from);
    copies.push_back(to);
    copies.push_back(rem);
  }
  dst.length = n;
  const int64_t id = next_id_++;
  seqs_.emplace(id, std::move(dst));
  return id;
}

const std::vector<int32_t>& KVManager::pages(int64_t seq) const { return get(seq).pages; }

int64_t KVManager::adopt(const std::vector<int32_t>& pages, int length) {
  const int n = static_cast<int>(pages.size());
  const bool ok = (n == 0 && length == 0) || (n > 0 && length > (n - 1) * page_size_ && length <= n * page_size_);
  if (!ok) throw std::invalid_argument("adopted length must end in the last page");
  for (int32_t p : pages) retain(p);
  Seq s;
  s.pages = pages;
  s.length = length;
  const int64_t id = next_id_++;
  seqs_.emplace(id, std::move(s));
  return id;
}

void KVManager::retain(int32_t page) {
  if (page < 0 || page >= static_cast<int32_t>(ref_.size()) || ref_[page] <= 0)
    throw std::logic_error("retain of a free page");
  ++ref_[page];
}

void KVManager::fill_table(const std::vector<int64_t>& seqs, int32_t* out, int stride) const {
  for (size_t r = 0; r < seqs.size(); ++r) {
    const Seq& s = get(seqs[r]);
    if (static_cast<int>(s.pages.size()) > stride) throw std::out_of_range("page table row too short");
    int32_t* row = out + r * stride;
    std::copy(s.pages.begin(), s.pages.end(), row);
    std::fill(row + s.pages.size(), row + stride, 0);
  }
}

}  // namespace osb
