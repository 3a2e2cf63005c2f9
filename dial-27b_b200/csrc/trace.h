// Layout of the opt-in decode-step timeline (DIAL_B200_TRACE=<csv>): a header
// of kTraceHeader words (records written, capacity) then records of
// kTraceWords words: [tag << 32 | CTA] and four %globaltimer stamps.
#pragma once

namespace dialb200 {

constexpr int kTraceHeader = 8, kTraceWords = 5;

}  // namespace dialb200
