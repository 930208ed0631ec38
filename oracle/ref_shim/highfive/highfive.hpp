// Type shim for HighFive (HDF5 C++ wrapper) -- TEST INFRASTRUCTURE ONLY.
//
// The reference's simulator declares HighFive types for its optional HDF5
// monitor output (src/simulate.h:85, src/io/variable_recorder.h:13,30).  libhdf5
// is not available here, so these do-nothing types let the reference's CPU
// integrator compile for the oracle; the harness runs with BufferEnable::NONE,
// so none of them is ever used for I/O.
#pragma once
#include <cstddef>
#include <initializer_list>
#include <string>
#include <vector>

namespace HighFive {

struct DataSpace {
    static const size_t UNLIMITED = (size_t)-1;
    DataSpace() {}
    DataSpace(std::initializer_list<size_t>, std::initializer_list<size_t>) {}
    DataSpace(const std::vector<size_t>&, const std::vector<size_t>&) {}
    std::vector<size_t> getDimensions() const { return {0}; }
};

struct Selection {
    template <class T>
    void write(const T*) {}
};

struct DataSet {
    DataSpace getSpace() const { return DataSpace(); }
    void resize(const std::vector<size_t>&) {}
    Selection select(const std::vector<size_t>&, const std::vector<size_t>&) { return Selection(); }
};

template <class T>
struct AtomicType {};

struct Chunking {
    Chunking(std::initializer_list<size_t>) {}
};

struct DataSetCreateProps {
    void add(const Chunking&) {}
};

struct Group {
    Group createGroup(const std::string&) { return Group(); }
    Group getGroup(const std::string&) { return Group(); }
    template <class T>
    DataSet createDataSet(const std::string&, const DataSpace&, const T&, const DataSetCreateProps&) {
        return DataSet();
    }
};

struct File {
    enum : unsigned { ReadOnly = 0, ReadWrite = 1, Create = 2, Truncate = 4 };
    File(const std::string&, unsigned) {}
    bool exist(const std::string&) const { return true; }
    Group createGroup(const std::string&) { return Group(); }
    Group getGroup(const std::string&) { return Group(); }
    template <class T>
    DataSet createDataSet(const std::string&, const DataSpace&, const T&, const DataSetCreateProps&) {
        return DataSet();
    }
};

}  // namespace HighFive
