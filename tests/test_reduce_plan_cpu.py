"""The split-row reduce plan (uk::plan_reduce in csrc/uk_plan.cuh) against the
fixed partial-sum capacity of uk_cuda_reduce_f32_noalloc (8192 floats).

The plan header is plain host C++, so this test compiles a small harness
against it with g++ (no GPU) and sweeps every row count that takes the split
plan (rows < 4 * sms) over long and ragged row lengths.  Bound: the split
plan needs rows * splits <= rows * ceil(8 sms / rows) < 12 sms partials, so
on a 148-SM B200 at most 1775 and never more than the capacity; on a part
with 1024 SMs some shapes would need more, which keeps the entry point's
refusal (UK_EINVAL) a live branch rather than dead code.
"""
import subprocess
from pathlib import Path

import pytest

PLAN = Path(__file__).resolve().parents[1] / "unikern_b200" / "csrc" / "uk_plan.cuh"
CAPACITY = 8192

HARNESS = r"""
#include <cstdio>
#include <cstdlib>
#include "uk_plan.cuh"
int main(int argc, char** argv) {
  const long long sms = atoll(argv[1]);
  const long long cols[] = {16384, 16385, 65536, 100003, 1 << 20, 5000001, 1LL << 22, 134217728, 1LL << 30};
  long long worst = 0, worst_rows = 0, worst_cols = 0;
  for (long long rows = 1; rows < 4 * sms; ++rows)
    for (long long c : cols) {
      const uk::ReducePlan p = uk::plan_reduce(rows, c, sms);
      if (p.mode != 3) continue;
      if (p.splits < 2 || p.chunk * p.splits < c || p.chunk * (p.splits - 1) >= c) return 2;
      if (rows * p.splits > worst) { worst = rows * p.splits; worst_rows = rows; worst_cols = c; }
    }
  printf("%lld %lld %lld\n", worst, worst_rows, worst_cols);
  return 0;
}
"""


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    d = tmp_path_factory.mktemp("plan")
    src = d / "plan_sweep.cpp"
    src.write_text(HARNESS)
    exe = d / "plan_sweep"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(PLAN.parent), str(src), "-o", str(exe)], check=True)
    return exe


def worst_need(exe, sms):
    r = subprocess.run([str(exe), str(sms)], capture_output=True, text=True)
    assert r.returncode == 0, "a split plan does not cover its row exactly"
    need, rows, cols = (int(v) for v in r.stdout.split())
    return need, rows, cols


def test_b200_split_plans_fit_the_no_alloc_scratch(harness):
    need, rows, cols = worst_need(harness, 148)
    assert need <= 12 * 148 - 1 == 1775
    assert need <= CAPACITY


def test_larger_parts_can_exceed_it(harness):
    # the entry point's size check is reachable on a big enough part
    assert worst_need(harness, 682)[0] <= CAPACITY
    assert worst_need(harness, 1024)[0] > CAPACITY
