/* CPU model of k_sample's windowed softmax-denominator sum (llmq_sample.cuh),
 * checked against the plain sequential float loop of sampler.c:74-80.
 *
 * The kernel evaluates ((0 + e_0) + e_1) + ... in windows: inside one binade of
 * the running sum s every rounded add moves s by round(e / u) grid steps
 * (u = the binade's spacing), except at exact half-way cases (round to even
 * on the parity of s / u) and at adds that may reach the next binade.  This
 * program restates the window logic sequentially (same step counts,
 * saturation, half-way list, early end of a window) and compares its result
 * bit for bit with the loop on random rows of eight kinds, and compares the
 * float form of the step count with the integer form.
 *
 * Usage: sampler_chain_check TRIALS STEP_CASES   (exit status 0 = all equal) */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define SAT (1u << 30)
#define WINDOW 8192
#define PER 8
#define HEAD 1024
#define TIE_CAP 512

typedef struct {
  uint32_t n, r;
  int tie;
} Step;

static uint32_t bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float flt(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t sat_add(uint32_t a, uint32_t b) { uint32_t s = a + b; return s < SAT ? s : SAT; }
static float pow2f(int x) { return x >= -126 ? flt((uint32_t)(x + 127) << 23) : flt(1u << (x + 149)); }

static Step step_int(uint32_t eb, int uexp) {
  const uint32_t ef = eb >> 23, me = ef ? ((eb & 0x7fffffu) | 0x800000u) : eb;
  const int d = (ef ? (int)ef - 150 : -149) - uexp;
  Step c = {0, 0, 0};
  if (d >= 0) {
    const unsigned long long n = d >= 40 ? SAT : ((unsigned long long)me << d);
    c.n = c.r = n >= SAT ? SAT : (uint32_t)n;
  } else if (d > -32) {
    const int sh = -d;
    const uint32_t rem = me & ((1u << sh) - 1u), half = 1u << (sh - 1);
    c.n = me >> sh;
    c.r = c.n + (rem > half);
    c.tie = rem == half;
  }
  return c;
}

static Step step_float(uint32_t eb, float inv_u) {
  volatile float t = flt(eb) * inv_u;
  const float n = floorf(t);
  volatile float fr = t - n;
  Step c;
  c.n = (uint32_t)fminf(n, 1073741824.0f);
  c.r = c.n + (fr > 0.5f);
  if (c.r > SAT) c.r = SAT;
  c.tie = fr == 0.5f;
  return c;
}

static float windowed_sum(const float *e, int V) {
  const int head = V < HEAD ? V : HEAD;
  volatile float s = 0.0f;
  for (int i = 0; i < head; i++) s = s + e[i];
  float cur = s;
  int base = head;
  static uint32_t thread_sum[WINDOW / PER];
  static int thread_ties[WINDOW / PER];
  static int tie_o[TIE_CAP];
  static uint32_t tie_p[TIE_CAP], tie_n[TIE_CAP], first_p, first_e;
  while (base < V) {
    const int len = V - base < WINDOW ? V - base : WINDOW;
    const uint32_t sb = bits(cur), sef = sb >> 23;
    const int uexp = sef ? (int)sef - 150 : -149;
    const uint32_t M = sef ? ((sb & 0x7fffffu) | 0x800000u) : sb;
    const int use_float = uexp >= -100 && uexp <= 0;
    const float inv_u = use_float ? pow2f(-uexp) : 0.0f;
    for (int t = 0; t < WINDOW / PER; t++) {
      uint32_t rs = 0;
      int ts = 0;
      for (int q = 0; q < PER; q++) {
        const int o = t * PER + q;
        const uint32_t eb = o < len ? bits(e[base + o]) : 0u;
        const Step c = use_float ? step_float(eb, inv_u) : step_int(eb, uexp);
        rs = sat_add(rs, c.r);
        ts += c.tie;
      }
      thread_sum[t] = rs;
      thread_ties[t] = ts;
    }
    uint32_t run = 0, total;
    int trun = 0, n_ties, jc = WINDOW;
    for (int t = 0; t < WINDOW / PER; t++) {
      uint32_t P = run;
      int Tc = trun;
      for (int q = 0; q < PER; q++) {
        const int o = t * PER + q;
        if (o >= len) continue;
        const Step c = use_float ? step_float(bits(e[base + o]), inv_u) : step_int(bits(e[base + o]), uexp);
        int flag = M + P + (uint32_t)Tc + c.r + 1u >= (1u << 24);
        if (c.tie) {
          if (Tc < TIE_CAP) { tie_o[Tc] = o; tie_p[Tc] = P; tie_n[Tc] = c.r; }
          else if (Tc == TIE_CAP) flag = 1;
        }
        if (flag && o < jc) { jc = o; first_p = P; first_e = bits(e[base + o]); }
        P = sat_add(P, c.r);
        Tc += c.tie;
      }
      run = sat_add(run, thread_sum[t]);
      trun += thread_ties[t];
    }
    total = run;
    n_ties = trun;
    if (jc > len) jc = len;
    const int nl = n_ties < TIE_CAP ? n_ties : TIE_CAP;
    uint32_t ups = 0;
    for (int i = 0; i < nl && tie_o[i] < jc; i++) ups += (M + tie_p[i] + ups + tie_n[i]) & 1u;
    const uint32_t Mn = M + (jc < len ? first_p : total) + ups;
    volatile float sn = (float)Mn * pow2f(uexp);
    if (jc < len) sn = sn + flt(first_e);
    cur = sn;
    base += jc < len ? jc + 1 : len;
  }
  return cur;
}

static uint64_t rs = 88172645463325252ull;
static uint64_t next64(void) { rs ^= rs << 13; rs ^= rs >> 7; rs ^= rs << 17; return rs; }
static double uni(void) { return (next64() >> 11) * (1.0 / 9007199254740992.0); }

int main(int argc, char **argv) {
  const int trials = argc > 1 ? atoi(argv[1]) : 800;
  const long step_cases = argc > 2 ? atol(argv[2]) : 20000000;
  int fails = 0;
  for (int trial = 0; trial < trials; trial++) {
    const int V = trial < 60 ? 1 + trial * 37 : (int)(uni() * 140000) + 1;
    float *e = malloc(sizeof(float) * (size_t)V);
    const int kind = trial % 8;
    const double sd = 0.5 + uni() * 4;
    for (int i = 0; i < V; i++) {
      const double g = sqrt(-2 * log(uni() + 1e-300)) * cos(6.283185307179586 * uni());
      float v;
      switch (kind) {
        case 0: v = expf((float)(g * sd) - 12.0f); break;                          /* smooth */
        case 1: v = (float)uni(); break;                                            /* uniform */
        case 2: v = ldexpf((float)(int)(uni() * 16), -(int)(uni() * 10)); break;   /* dyadic: ties */
        case 3: v = expf((float)(g * 60)); if (v > 1) v = 1; break;                 /* wide */
        case 4: v = (i % 1000 == 0) ? 1.0f : ldexpf(1.0f, -24 - (int)(uni() * 4)); break;
        case 5: v = (float)(uni() < 0.001 ? 1.0 : uni() * 1e-7); break;
        case 6: v = ldexpf((float)uni(), -140); break;                               /* subnormal */
        default: v = (i == 0) ? 1e-30f : (float)uni() * 0.25f; break;
      }
      e[i] = v;
    }
    if (trial % 5 == 0) e[(int)(uni() * V)] = 1.0f;
    volatile float s = 0.0f;
    for (int i = 0; i < V; i++) s = s + e[i];
    const float w = windowed_sum(e, V);
    if (bits(w) != bits(s)) {
      if (fails++ < 5) printf("sum mismatch: trial %d kind %d V %d: loop %a windows %a\n", trial, kind, V, s, w);
    }
    free(e);
  }
  long step_fails = 0;
  for (long i = 0; i < step_cases; i++) {
    uint32_t eb = (uint32_t)next64() & 0x3fffffffu;
    if (eb > 0x3f800000u) eb = (uint32_t)(next64() % 0x3f800001u);
    if ((i & 7) == 0) eb &= ~((1u << (next64() % 24)) - 1u);
    const int uexp = -(int)(next64() % 101);
    const Step a = step_int(eb, uexp), b = step_float(eb, pow2f(-uexp));
    const uint32_t an = a.n > SAT ? SAT : a.n;
    if (a.r != b.r || a.tie != b.tie || an != b.n) {
      if (step_fails++ < 5) printf("step mismatch: e %08x uexp %d\n", eb, uexp);
    }
  }
  printf("%d of %d sums differ; %ld of %ld step counts differ\n", fails, trials, step_fails, step_cases);
  return fails || step_fails;
}
