// mc_tables.h -- marching-cubes case table (the standard VTK table, in the
// triangle order the reference emits), encoded compactly.
//
// Case c (bit b set <=> corner b is above the isovalue) lists its triangles
// as a string of hexadecimal edge ids, three per triangle.  Corners are
// 0:(i,j,k) 1:(i+1,j,k) 2:(i+1,j+1,k) 3:(i,j+1,k) and 4..7 the same at k+1;
// edges are 0:(0,1) 1:(1,2) 2:(3,2) 3:(0,3) 4:(4,5) 5:(5,6) 6:(7,6) 7:(4,7)
// 8:(0,4) 9:(1,5) 10:(3,7) 11:(2,6).  The content has to equal the
// reference's table (packages/tack-vis/src/tack/algorithms/flying_edges.py:33-306)
// entry for entry: triangle order and vertex order decide the output bytes.
#pragma once
#include <stdint.h>

// X("edges") once per case, cases 0..255 in order.
#define TKMC_CASE_LIST(X) \
  X("") X("038") X("091") X("138918") X("1b2") X("0381b2") X("9b2092") X("23828bb89") \
  X("32a") X("02a80a") X("1092a3") X("12a1a99a8") X("31ba3b") X("01b0b88ba") X("30939aa9b") X("9b8ba8") \
  X("487") X("403743") X("091874") X("491417713") X("1b2874") X("3743401b2") X("9b2920874") X("29b279237749") \
  X("87432a") X("a74a42240") X("9108742a3") X("4a79a492a912") X("31b3ba748") X("1ba1a414074a") X("4879a09baa30") X("4a749a9ba") \
  X("945") X("945038") X("045105") X("845853351") X("1b2945") X("3801b2459") X("5b2524420") X("25b352345384") \
  X("9452a3") X("02a0a8459") X("0450512a3") X("2512852a8458") X("ba3b31945") X("45901881b8ba") X("5045a05baa30") X("5845b8ba8") \
  X("987597") X("903935537") X("087071175") X("135375") X("987975b21") X("b21905503537") X("820852875b25") X("25b235375") \
  X("75979832a") X("9759279022a7") X("2a3081187175") X("a12a71751") X("985875b31ba3") X("50759070a1b0a0b") X("a0ba30b05870507") X("a5b75a") \
  X("b56") X("03856b") X("91056b") X("13818956b") X("156216") X("156162380") X("956960062") X("589528562382") \
  X("2a3b56") X("a80a02b56") X("0912a356b") X("56b12992a9a8") X("6a3635531") X("0a805a01556a") X("36a063056095") X("6956a9a89") \
  X("56b487") X("4034376b5") X("10956b874") X("b56179137749") X("621615487") X("152562340374") X("874950056062") X("793749392569296") \
  X("32a748b56") X("56b4274022a7") X("0914872a356b") X("91292a9a474a56b") X("87435a31556a") X("5a156a1a074a0a4") X("095056063a36874") X("6956a949779a") \
  X("b946b4") X("46b4b9038") X("b10b06604") X("8138618466b1") X("194142246") X("380192294246") X("042462") X("823842462") \
  X("b94b46a32") X("0282a84b946b") X("32a0610466b1") X("6146b14182a181a") X("946963931a36") X("81a801a16941614") X("36a306046") X("684a86") \
  X("76b7b88b9") X("03707b0b96b7") X("b7617b187108") X("b76b17137") X("162186198876") X("296219697039793") X("708760620") X("723627") \
  X("2a3b86b98876") X("2702a70796b797b") X("10818717b6b72a3") X("a12a71b16617") X("869876961a36163") X("019a76") X("70876030aa06") X("76a") \
  X("7a6") X("380a67") X("091a67") X("891813a67") X("b2167a") X("1b238067a") X("20929b67a") X("67a23bb38b89") \
  X("732672") X("780706602") X("267273091") X("126168189867") X("b67b71173") X("b671b7178180") X("0730b709b67b") X("7b678b89b") \
  X("648a68") X("3a6360064") X("8a6864910") X("964936913a63") X("64868a21b") X("1b23a00a6064") X("48a4a609229b") X("b39b23934a63436") \
  X("832824426") X("024426") X("109243264483") X("149124264") X("83181686461b") X("b01b60640") X("43648363b093b39") X("b4964b") \
  X("4597a6") X("038459a67") X("5105047a6") X("a67843345351") X("945b217a6") X("67a1b2038459") X("7a65b44b2420") X("384345352b25a67") \
  X("732726594") X("945068026678") X("326367105504") X("682678281458185") X("945b61167173") X("1b6167170807945") X("4b045b0b367b3b7") X("7b678b5b44b8") \
  X("65969aa98") X("3a6036065059") X("08a0a50515a6") X("63a653513") X("1b29a598aa65") X("03a0a60695961b2") X("a58a65850b25052") X("63a65323bb35") \
  X("598582526328") X("965906026") X("185108586328682") X("165261") X("1631b6368596869") X("b01b60905506") X("0835b6") X("b65") \
  X("ab57a5") X("ab5a57803") X("57a5ab109") X("b57b7a918813") X("a21a17715") X("0381721577a2") X("95797292027a") X("7257a2529382928") \
  X("2b5253357") X("802825857b52") X("91053b57332b") X("928912827b52725") X("153357") X("078017157") X("930953573") X("978579") \
  X("54858bb8a") X("54050a5aba03") X("0918b48abb54") X("b4ab54a43914341") X("21525828a485") X("0a403a4a521a5a1") X("05209525a485a58") X("95423a") \
  X("2b5325354348") X("52b542402") X("32b3b5358485091") X("52b542129924") X("854835315") X("054150") X("854835950053") X("954") \
  X("47a4a99ab") X("03847997a9ab") X("1ab14a1047a4") X("34138414b7a4b4a") X("47a94a9a2921") X("94797a9a121a038") X("a47a24204") X("a47a24843342") \
  X("2b9297273794") X("97b947b72807270") X("3b732b7b410b4b0") X("12b847") X("419471731") X("419471018817") X("430734") X("478") \
  X("98bb8a") X("3903a9ab9") X("0b108b8ab") X("3b1ab3") X("1a219a98a") X("3903a919229a") X("0a28a0") X("3a2") \
  X("2832b8b98") X("92b029") X("2832b808118b") X("12b") X("183981") X("019") X("083") X("") \
  /* end */

namespace tkmc {

#define TKMC_CASE_STR(s) s,
static const char* const kCaseEdges[256] = {TKMC_CASE_LIST(TKMC_CASE_STR)};
#undef TKMC_CASE_STR

// Edge e joins corners kEdgeCorners[2e] and kEdgeCorners[2e+1].
static const int kEdgeCorners[24] = {0, 1, 1, 2, 3, 2, 0, 3, 4, 5, 5, 6,
                                     7, 6, 4, 7, 0, 4, 1, 5, 3, 7, 2, 6};

constexpr int hex_nibble(char ch) {
  return (ch >= '0' && ch <= '9') ? ch - '0' : ch - 'a' + 10;
}

// One case string -> packed word (see pack_case_table); usable in constant
// initialisers of device tables.
constexpr uint64_t pack_case(const char* s) {
  uint64_t w = 0;
  int n = 0;
  while (s[n]) {
    w |= (uint64_t)hex_nibble(s[n]) << (4 * n);
    ++n;
  }
  return w | ((uint64_t)(n / 3) << 60);
}

// Packed form used on the device: nibbles 0..14 hold the edge ids of up to
// five triangles in order, nibble 15 holds the triangle count.
inline void pack_case_table(uint64_t out[256]) {
  for (int c = 0; c < 256; ++c) out[c] = pack_case(kCaseEdges[c]);
}

// Unpacked form of the reference: 16 entries per case, -1 padded.
inline void unpack_tri_table(int32_t tri_table[4096], int32_t num_tris[256]) {
  for (int c = 0; c < 256; ++c) {
    int n = 0;
    for (const char* p = kCaseEdges[c]; *p; ++p, ++n)
      if (tri_table) tri_table[c * 16 + n] = hex_nibble(*p);
    if (tri_table)
      for (int t = n; t < 16; ++t) tri_table[c * 16 + t] = -1;
    if (num_tris) num_tris[c] = n / 3;
  }
}

}  // namespace tkmc
