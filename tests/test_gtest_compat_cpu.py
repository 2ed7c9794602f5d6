"""The gtest-compatible harness (tests/gtest_compat) that lets the
reference's own unit tests compile without GoogleTest: it runs the
reference's tests green against the reference's CPU library, and it reports
failures (EXPECT_* counts and continues, ASSERT_* leaves the test, an
uncaught exception fails the test, the exit status is 1)."""
import os
import subprocess
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GTC = os.path.join(ROOT, "tests", "gtest_compat")
REF_TESTS_CPU = os.path.join(ROOT, "oracle", "_ref", "ref_tests_cpu")


def test_reference_unit_tests_pass_on_reference_library():
    if not os.path.exists(REF_TESTS_CPU):
        pytest.skip("oracle/_ref/ref_tests_cpu not built (it needs the reference sources)")
    r = subprocess.run([REF_TESTS_CPU], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:]
    assert "[  PASSED  ] 22 tests." in r.stdout


def test_harness_reports_failures(tmp_path):
    src = tmp_path / "t.cpp"
    src.write_text(textwrap.dedent("""
        #include <stdexcept>
        #include <vector>
        #include <gtest/gtest.h>
        static int after_assert = 0;
        TEST(Self, Passes) {
            EXPECT_EQ(2 + 2, 4);
            EXPECT_NEAR(1.0, 1.05, 0.1);
            EXPECT_FLOAT_EQ(0.1f + 0.2f, 0.3f);
            EXPECT_LE(1, 2);
            EXPECT_TRUE(true) << "unused";
            EXPECT_THROW(throw std::invalid_argument("x"), std::invalid_argument);
            EXPECT_THROW(std::vector<int>({1, 2}).at(5), std::out_of_range);
        }
        TEST(Self, ExpectFails) {
            EXPECT_EQ(1, 2) << "streamed note";
            EXPECT_FLOAT_EQ(1.0f, 1.001f);
            EXPECT_THROW((void)0, std::invalid_argument);
        }
        TEST(Self, AssertLeaves) {
            ASSERT_TRUE(false);
            after_assert = 1;
        }
        TEST(Self, Throws) { throw std::runtime_error("boom"); }
        TEST(Self, AssertDidLeave) { EXPECT_EQ(after_assert, 0); }
    """))
    exe = tmp_path / "t"
    subprocess.run(["g++", "-std=c++20", "-I", GTC, "-o", str(exe), str(src),
                    os.path.join(GTC, "gtest_main.cpp")], check=True, timeout=120)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    out = r.stdout
    assert "[       OK ] Self.Passes" in out
    assert "[  FAILED  ] Self.ExpectFails" in out and "streamed note" in out
    assert "throws nothing" in out
    assert "[  FAILED  ] Self.AssertLeaves" in out
    assert "[  FAILED  ] Self.Throws" in out and "boom" in out
    assert "[       OK ] Self.AssertDidLeave" in out
    assert "[  FAILED  ] 3 tests." in out
    r = subprocess.run([str(exe), "--gtest_filter=Self.Passes"], capture_output=True, text=True,
                       timeout=60)
    assert r.returncode == 0 and "[  PASSED  ] 1 tests." in r.stdout
