// CPU checks of miag_moe's host-side transfer pieces (host_copy.h): the copy
// threads reproduce memcpy for any size and worker count, including calls
// issued back to back and after the workers have gone to sleep, and the
// piece split covers a batch exactly once in increasing, non-empty pieces.
#include "../../motoria_b200/csrc/host_copy.h"

#include <cstdio>
#include <random>

static int check_pool() {
    std::mt19937_64 g(7);
    for (int workers : {0, 1, 2, 5, 7}) {
        miag::CopyPool pool(workers);
        for (int it = 0; it < 200; it++) {
            size_t n = (size_t)(g() % (6u << 20)) + 1;
            if (it % 7 == 0) n = (size_t)(g() % 4096) + 1;  // below the split threshold
            std::vector<unsigned char> a(n), b(n, 0xA5);
            for (size_t i = 0; i < n; i++) a[i] = (unsigned char)(g() >> 56);
            const size_t off = g() % 64;  // unaligned starts
            if (off < n) {
                pool.copy(b.data() + off, a.data() + off, n - off);
                if (memcmp(a.data() + off, b.data() + off, n - off) != 0) {
                    printf("copy mismatch: workers %d, bytes %zu, offset %zu\n", workers, n, off);
                    return 1;
                }
                for (size_t i = 0; i < off; i++)
                    if (b[i] != 0xA5) {
                        printf("write before the destination: workers %d\n", workers);
                        return 1;
                    }
            }
            if (it % 50 == 49) std::this_thread::sleep_for(std::chrono::milliseconds(2));  // workers sleep
        }
    }
    return 0;
}

static int check_pieces() {
    for (int n = 1; n < 40000; n += (n < 300 ? 1 : 37)) {
        for (int chunks = 1; chunks <= 16; chunks++) {
            const std::vector<int> b = miag::piece_bounds(n, chunks);
            const int pieces = (int)b.size() - 1;
            if (b.front() != 0 || b.back() != n || pieces < 1 || pieces > chunks) {
                printf("bad split: n %d, chunks %d, %d pieces\n", n, chunks, pieces);
                return 1;
            }
            for (int k = 0; k < pieces; k++)
                if (b[k + 1] <= b[k]) {
                    printf("empty piece: n %d, chunks %d, piece %d\n", n, chunks, k);
                    return 1;
                }
        }
    }
    const std::vector<int> want{0, 512, 2048, 3584, 4096};  // config 5, four pieces
    if (miag::piece_bounds(4096, 4) != want) {
        printf("config 5 split changed\n");
        return 1;
    }
    return 0;
}

int main() {
    if (check_pool() || check_pieces()) return 1;
    printf("ok\n");
    return 0;
}
