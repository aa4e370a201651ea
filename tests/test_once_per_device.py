"""The launchers' one-time kernel-attribute set-up is kept per device.

Kernel attributes (dynamic shared-memory limit, carveout) belong to the
device that is current when they are set, and hpc_device_init selects the
device per host thread, so one process may drive several devices.  Each
launcher therefore records, one bit per device, where its set-up succeeded
(heliopause_b200/csrc/hc_once.h).  The helper is host-only C++: this test
compiles it with g++ and checks its bookkeeping without a GPU.
"""
import shutil
import subprocess
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parents[1] / "heliopause_b200" / "csrc"

DRIVER = r"""
#include <cstdio>
#include <thread>
#include <vector>
#include "hc_once.h"

static int calls = 0;
static int fail_next = 0;
static int set() {
  ++calls;
  if (fail_next) { --fail_next; return 7; }
  return 0;
}

#define CHECK(c) do { if (!(c)) { std::printf("FAIL line %d: %s\n", __LINE__, #c); return 1; } } while (0)

int main() {
  std::atomic<uint64_t> done{0};
  // once per device
  CHECK(hc::once_per_device<int>(done, 0, set) == 0 && calls == 1);
  CHECK(hc::once_per_device<int>(done, 0, set) == 0 && calls == 1);
  CHECK(hc::once_per_device<int>(done, 1, set) == 0 && calls == 2);
  CHECK(hc::once_per_device<int>(done, 1, set) == 0 && calls == 2);
  CHECK(hc::once_per_device<int>(done, 63, set) == 0 && calls == 3);
  CHECK(done.load() == ((uint64_t(1) << 63) | 3u));
  // a failed set-up is returned and not recorded; the next call retries
  fail_next = 1;
  CHECK(hc::once_per_device<int>(done, 5, set) == 7 && calls == 4);
  CHECK((done.load() & (uint64_t(1) << 5)) == 0);
  CHECK(hc::once_per_device<int>(done, 5, set) == 0 && calls == 5);
  CHECK(hc::once_per_device<int>(done, 5, set) == 0 && calls == 5);
  // devices without a bit run the set-up every time and mark nothing
  const uint64_t before = done.load();
  CHECK(hc::once_per_device<int>(done, 64, set) == 0 && calls == 6);
  CHECK(hc::once_per_device<int>(done, 64, set) == 0 && calls == 7);
  CHECK(hc::once_per_device<int>(done, -1, set) == 0 && calls == 8);
  CHECK(done.load() == before);
  // concurrent first calls on one device: the set-up runs at least once,
  // every caller sees success, and the bit ends up set
  std::atomic<uint64_t> shared{0};
  std::atomic<int> runs{0}, bad{0};
  std::vector<std::thread> ts;
  for (int i = 0; i < 8; ++i)
    ts.emplace_back([&] {
      const int e = hc::once_per_device<int>(shared, 2, [&] { runs.fetch_add(1); return 0; });
      if (e != 0) bad.fetch_add(1);
    });
  for (auto& t : ts) t.join();
  CHECK(bad.load() == 0 && runs.load() >= 1 && runs.load() <= 8);
  CHECK(shared.load() == (uint64_t(1) << 2));
  const int after = runs.load();
  CHECK(hc::once_per_device<int>(shared, 2, [&] { runs.fetch_add(1); return 0; }) == 0 && runs.load() == after);
  std::printf("ok\n");
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_once_per_device_bookkeeping(tmp_path):
    src = tmp_path / "once_driver.cpp"
    exe = tmp_path / "once_driver"
    src.write_text(DRIVER)
    subprocess.run(["g++", "-std=c++17", "-O1", "-pthread", f"-I{CSRC}", str(src), "-o", str(exe)], check=True,
                   capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr


def test_launchers_keep_no_process_wide_attribute_flag():
    # every launcher's attribute set-up goes through the per-device helper
    offenders = []
    for f in sorted(CSRC.glob("*.cu")):
        for n, line in enumerate(f.read_text().splitlines(), 1):
            if "static bool attr" in line:
                offenders.append(f"{f.name}:{n}")
    assert not offenders, offenders
