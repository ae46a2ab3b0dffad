/*
 * Deterministic transcendental functions for the oracle.  TEST INFRASTRUCTURE ONLY.
 *
 * The task-aligned assigner (DetectionLoss.cs:48-68) ranks anchors by
 * sigmoid(logit)^0.5 * CIoU^6, where the decoded boxes come from a DFL softmax
 * (DetectionLoss.cs:37-43) and CIoU uses atan (DetectionLoss.cs:180).  To make the
 * assignment reproducible bit for bit between this CPU restatement and the CUDA
 * kernels, exp and atan are evaluated here from published methods using only
 * IEEE-754 double operations with explicit fma:
 *   exp : Cody-Waite reduction by ln 2 (two-part split of ln 2, as in fdlibm),
 *         Taylor series of degree 13 on |r| <= ln2/2, exact scaling by 2^k.
 *   atan: reduction to [0,1] by atan(x) = pi/2 - atan(1/x), then to |t| <= tan(pi/12)
 *         by atan(x) = pi/6 + atan((x*sqrt3 - 1)/(x + sqrt3)), odd Taylor series to t^25.
 * Float results are these double values rounded once, so they are within one ulp of
 * the platform libm that the reference calls.  Compiled with -ffp-contract=off.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include "syo.h"

static const double LOG2E = 1.4426950408889634074;
static const double LN2_HI = 6.93147180369123816490e-01; /* upper bits of ln 2, k*LN2_HI exact */
static const double LN2_LO = 1.90821492927058770002e-10; /* ln 2 - LN2_HI */

double syo_exp_d(double x)
{
    if (x != x) return x;
    if (x > 200.0) x = 200.0;       /* far beyond float range; double stays finite */
    if (x < -200.0) x = -200.0;
    double k = nearbyint(x * LOG2E);
    double r = fma(-k, LN2_HI, x);
    r = fma(-k, LN2_LO, r);
    double p = 1.0 / 6227020800.0;  /* 1/13! */
    p = fma(p, r, 1.0 / 479001600.0);
    p = fma(p, r, 1.0 / 39916800.0);
    p = fma(p, r, 1.0 / 3628800.0);
    p = fma(p, r, 1.0 / 362880.0);
    p = fma(p, r, 1.0 / 40320.0);
    p = fma(p, r, 1.0 / 5040.0);
    p = fma(p, r, 1.0 / 720.0);
    p = fma(p, r, 1.0 / 120.0);
    p = fma(p, r, 1.0 / 24.0);
    p = fma(p, r, 1.0 / 6.0);
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    int64_t e = (int64_t)k + 1023;  /* |k| <= 289, always a normal double */
    uint64_t bits = (uint64_t)e << 52;
    double scale;
    memcpy(&scale, &bits, sizeof scale);
    return p * scale;
}

float syo_expf(float x) { return (float)syo_exp_d((double)x); }

static const double PI_2 = 1.57079632679489661923;
static const double PI_6 = 0.52359877559829887308;
static const double SQRT3 = 1.73205080756887729353;
static const double TAN_PI_12 = 0.26794919243112270647;

double syo_atan_d(double x)
{
    if (x != x) return x;
    int negative = x < 0;
    if (negative) x = -x;
    int inverted = 0;
    if (x > 1.0) {
        inverted = 1;
        x = 1.0 / x;
    }
    double offset = 0.0;
    if (x > TAN_PI_12) {
        x = (x * SQRT3 - 1.0) / (x + SQRT3);
        offset = PI_6;
    }
    /* atan(t) = t * (1 - t^2/3 + t^4/5 - ... + t^24/25) */
    double t2 = x * x;
    double p = 1.0 / 25.0;
    p = fma(p, t2, -1.0 / 23.0);
    p = fma(p, t2, 1.0 / 21.0);
    p = fma(p, t2, -1.0 / 19.0);
    p = fma(p, t2, 1.0 / 17.0);
    p = fma(p, t2, -1.0 / 15.0);
    p = fma(p, t2, 1.0 / 13.0);
    p = fma(p, t2, -1.0 / 11.0);
    p = fma(p, t2, 1.0 / 9.0);
    p = fma(p, t2, -1.0 / 7.0);
    p = fma(p, t2, 1.0 / 5.0);
    p = fma(p, t2, -1.0 / 3.0);
    double result = fma(x * t2, p, x);
    result += offset;
    if (inverted) result = PI_2 - result;
    return negative ? -result : result;
}

float syo_atanf(float x) { return (float)syo_atan_d((double)x); }

/* HeadOperations.Sigmoid (HeadOperations.cs:222) with syo_expf in place of MathF.Exp. */
float syo_sigmoid(float value)
{
    if (value >= 0) return 1.0f / (1.0f + syo_expf(-value));
    float e = syo_expf(value);
    return e / (1.0f + e);
}

/* MathF.Pow(x, 6) (DetectionLoss.cs:63): exact-ish double product rounded once to float. */
float syo_pow6(float x)
{
    double t = (double)x;
    double t2 = t * t;
    double t4 = t2 * t2;
    return (float)(t4 * t2);
}
