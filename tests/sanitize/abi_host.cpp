// abi_host.cpp — drives the host side of libqcache (sequence and page
// bookkeeping, the decode-step protocol, the reference prefix rule, the hashed
// prefix table and its refcounts, argument errors) on a host-only context,
// linked against a build of the library instrumented with AddressSanitizer
// and UndefinedBehaviorSanitizer (tests/sanitize/Makefile).  Any memory error
// or undefined behaviour aborts with a report; a failed expectation exits 1.
// No GPU is used: every device call of a host-only context returns
// QC_ERR_NODEVICE, which is checked too.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../../include/qbfp8.h"
#include "../../include/qcache.h"
#include "../../include/qsample.h"

static int failures = 0;
#define EXPECT(cond)                                                        \
  do {                                                                      \
    if (!(cond)) {                                                          \
      std::fprintf(stderr, "%s:%d: expectation failed: %s\n", __FILE__,     \
                   __LINE__, #cond);                                        \
      ++failures;                                                           \
    }                                                                       \
  } while (0)

static std::vector<int32_t> pages(qc_ctx* q, int32_t s) {
  std::vector<int32_t> p(64);
  int32_t n = 0;
  EXPECT(qc_seq_pages(q, s, p.data(), (int32_t)p.size(), &n) == QC_OK);
  p.resize(n);
  return p;
}

static void step(qc_ctx* q, int32_t s, int32_t token) {
  EXPECT(qc_decode_begin(q, &s, 1, &token, nullptr) == QC_OK);
  EXPECT(qc_decode_end(q) == QC_OK);
}

int main() {
  qc_config cfg = {8, 24, 4, 16, 4096, 4, 4, 0};
  qc_ctx* q = nullptr;
  EXPECT(qc_create(&cfg, QC_DEVICE_NONE, &q) == QC_OK && q);

  // bad configurations and arguments fail without touching memory
  qc_config bad = cfg;
  bad.max_seqs = 0;
  qc_ctx* q2 = nullptr;
  EXPECT(qc_create(&bad, QC_DEVICE_NONE, &q2) != QC_OK && !q2);
  EXPECT(qc_create(nullptr, QC_DEVICE_NONE, &q2) != QC_OK);
  EXPECT(qc_seq_reserve(q, 99, 10) != QC_OK);
  EXPECT(qc_decode_end(q) != QC_OK);

  // slots and pages: allocation, rollback on exhaustion, reuse after free
  int32_t a = -1, b = -1;
  EXPECT(qc_seq_alloc(q, &a) == QC_OK && qc_seq_alloc(q, &b) == QC_OK);
  EXPECT(qc_seq_reserve(q, a, 64 * 12 + 1) == QC_OK);   // 13 pages of 16
  EXPECT(pages(q, a).size() == 13);
  EXPECT(qc_seq_reserve(q, b, 64 * 3 + 1) == QC_ERR_OOM); // needs 4, 3 left
  EXPECT(pages(q, b).empty());
  EXPECT(qc_seq_free(q, a) == QC_OK);
  EXPECT(qc_seq_reserve(q, b, 64 * 16) == QC_OK && pages(q, b).size() == 16);
  EXPECT(qc_seq_reset(q, b, nullptr) == QC_OK && pages(q, b).empty());

  // decode protocol, a page mapped at each boundary, device calls refused
  int32_t s = -1;
  EXPECT(qc_seq_alloc(q, &s) == QC_OK);
  for (int t = 0; t < 130; ++t) step(q, s, 1000 + t);
  int32_t len = 0;
  EXPECT(qc_seq_len(q, s, &len) == QC_OK && len == 130 && pages(q, s).size() == 3);
  EXPECT(qc_decode_begin(q, &s, 1, nullptr, nullptr) == QC_OK);
  EXPECT(qc_attn_decode(q, 0, nullptr, nullptr, nullptr) != QC_OK);
  EXPECT(qc_decode_begin(q, &s, 1, nullptr, nullptr) != QC_OK);  // step already open
  EXPECT(qc_decode_abort(q) == QC_OK);
  int32_t twice[2] = {s, s};
  EXPECT(qc_decode_begin(q, twice, 2, nullptr, nullptr) != QC_OK);

  // the reference's prefix rule (src/engine.cpp:4058-4080): 3 tokens cached
  EXPECT(qc_seq_reset(q, s, nullptr) == QC_OK);
  for (int t = 0; t < 3; ++t) step(q, s, 1000 + t);
  const int32_t prompt[5] = {1000, 1001, 1002, 9, 9};
  int32_t plen = -1;
  EXPECT(qc_seq_match_prefix(q, s, prompt, 5, &plen, nullptr) == QC_OK && plen == 3);
  EXPECT(qc_seq_match_prefix(q, s, prompt, 3, &plen, nullptr) == QC_OK && plen == 0);

  // hashed prefix table: insert, lookup with token verification, restore,
  // copy-on-write tail, refcounted release
  std::vector<int32_t> pre(150);
  for (int i = 0; i < 150; ++i) pre[i] = (i * 7919) % 248320;
  int32_t p = -1;
  EXPECT(qc_seq_alloc(q, &p) == QC_OK && qc_seq_reserve(q, p, 150) == QC_OK);
  int32_t e = -1;
  EXPECT(qc_prefix_insert(q, p, pre.data(), 150, &e, nullptr) == QC_OK && e >= 0);
  std::vector<int32_t> req(pre);
  req.push_back(3);
  int32_t matched = 0, ent = -1;
  EXPECT(qc_prefix_lookup(q, req.data(), (int32_t)req.size(), &matched, &ent) == QC_OK);
  EXPECT(matched == 150 && ent == e);
  req[10] ^= 1;
  EXPECT(qc_prefix_lookup(q, req.data(), (int32_t)req.size(), &matched, &ent) == QC_OK);
  EXPECT(matched == 0 && ent == -1);
  std::vector<uint64_t> h(2);
  EXPECT(qc_prefix_page_hashes(pre.data(), 150, h.data()) == QC_OK && h[0] != h[1]);
  EXPECT(qc_prefix_release(q, e) == QC_OK);
  EXPECT(qc_prefix_release(q, 1234) != QC_OK);

  {  // an exhausted pool or snapshot table leaves every sequence as it was
    qc_config small = {8, 24, 4, 7, 4096, 4, 1, 0};
    qc_ctx* r = nullptr;
    EXPECT(qc_create(&small, QC_DEVICE_NONE, &r) == QC_OK && r);
    int32_t u = -1, v = -1, w = -1;
    EXPECT(qc_seq_alloc(r, &u) == QC_OK && qc_seq_alloc(r, &v) == QC_OK &&
           qc_seq_alloc(r, &w) == QC_OK);
    EXPECT(qc_seq_reserve(r, u, 128) == QC_OK && qc_seq_reserve(r, v, 128) == QC_OK);
    EXPECT(qc_seq_reserve(r, w, 2 * 64) == QC_OK);          // 7 - 6 = 1 page free
    const std::vector<int32_t> pu = pages(r, u), pv = pages(r, v);
    int32_t both[2] = {u, v};
    EXPECT(qc_decode_begin(r, both, 2, nullptr, nullptr) == QC_ERR_OOM);
    EXPECT(pages(r, u) == pu && pages(r, v) == pv);
    step(r, v, 5);                                           // one page: fits
    EXPECT(pages(r, v).size() == 3 && pages(r, u) == pu);
    std::vector<int32_t> toks(129);
    for (int32_t i = 0; i < 129; ++i) toks[i] = i;
    int32_t e1 = -1, e2 = -1;
    EXPECT(qc_prefix_insert(r, u, toks.data(), 128, &e1, nullptr) == QC_OK);
    EXPECT(qc_prefix_insert(r, v, toks.data(), 129, &e2, nullptr) == QC_ERR_OOM);  // no slot
    EXPECT(qc_prefix_release(r, e1) == QC_OK);
    // a slot again, but the entry's tail page cannot be had: nothing is taken
    EXPECT(qc_prefix_insert(r, v, toks.data(), 129, &e2, nullptr) == QC_ERR_OOM);
    EXPECT(qc_prefix_insert(r, u, toks.data(), 128, &e1, nullptr) == QC_OK);
    EXPECT(qc_prefix_release(r, e1) == QC_OK);
    qc_destroy(r);
  }

  // peer-memory split-K needs a device; bad ranks are rejected first
  char handle[QC_P2P_HANDLE_BYTES];
  EXPECT(qc_p2p_create(q, 2, 0, handle) == QC_ERR_NODEVICE);
  EXPECT(qc_p2p_create(q, 1, 0, handle) == QC_ERR_ARG);
  EXPECT(qc_p2p_open(q, 1, handle) == QC_ERR_NODEVICE);
  EXPECT(qc_attn_combine_p2p(q, 0, nullptr, nullptr, nullptr) == QC_ERR_ARG);

  // the other headers' entry points reject missing arguments
  EXPECT(qc_bfp8_gemv(nullptr, nullptr, 1, nullptr, nullptr) == QC_ERR_ARG);
  EXPECT(qc_bfp8_packed_bytes(33, 32) == -1);
  EXPECT(qc_sample(nullptr, 10, 10, 1, 0.0f, 0.9f, nullptr, nullptr, nullptr) == QC_ERR_ARG);

  qc_destroy(q);
  qc_destroy(nullptr);
  if (failures) {
    std::fprintf(stderr, "%d expectation(s) failed\n", failures);
    return 1;
  }
  std::printf("host ABI under ASan/UBSan: ok\n");
  return 0;
}
